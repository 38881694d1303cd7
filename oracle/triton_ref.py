"""The reference's own Triton drop-ins, run beside this library on the same GPU.

Test and benchmark infrastructure only, like the rest of ``oracle/``: nothing
in ``kernelproblems_b200`` imports it.  It serves two legs:

* ``tests/test_gpu_triton_ref.py`` checks each reference kernel against the
  CPU oracle on the same seeded inputs, and
* ``bench.py`` times each reference kernel beside this library's drop-in for
  the same problem (same inputs, same CUDA-graph replay and event timing).

``fetch(reference_root)`` copies the eight ``optimized_kernel.py`` files of
the problems the five benchmark configurations come from into
``oracle/_ref/triton/`` (git-ignored; the directory travels to the GPU box
with the working tree, the reference checkout does not).  Three of them fix
their sizes in the host wrapper; each is patched to take the size from its
inputs instead, so it runs at the configuration's size.  The kernels
themselves are not changed.  Every patch is an exact text replacement that
must match once, listed in PATCHES:

  v8/c8c60d8f7015  RoPE fwd    S = 8192 (optimized_kernel.py:50) -> tokens of the positions input
  v7/bfe872e373e4  RoPE bwd q  S = 8192 (:58) and the [8192, 4096] output (:64) -> S of the input
  v7/5c65f62b0422  RoPE bwd k  S = 8192 (:50) -> S of the input
  v8/7884328a5557  add+norm    M = 8192, N = 4096 (:38-39) -> from the inputs' shapes
  v7/7f544ceb2120  norm bwd    M = 8192, N = 4096 (:74-75), BLOCK_N = 4096 (:85) -> from the
                               inputs (BLOCK_N the next power of two of N, as the kernel masks
                               columns by N)

Unpatched: v8/f4e9e58fef73 (RMSNorm fwd), v7/45990c83cfd6 (RMSNorm bwd),
v7/1e49beb8a123 (embedding fwd, D = 4096 as in the configuration) and
v7/a12a160cb11b (embedding bwd, vocab 128256 as in the configuration).
"""
from __future__ import annotations

import hashlib
import importlib.util
import json
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT_DIR = HERE / "_ref" / "triton"

# problem -> [(original text, replacement)]
PATCHES: dict[str, list[tuple[str, str]]] = {
    "v8/c8c60d8f7015": [
        ("    S = 8192\n", "    S = arg586_1.numel()\n"),
    ],
    "v7/bfe872e373e4": [
        ("    S = 8192\n", "    S = getitem_641.shape[2]\n"),
        ("    out = torch.empty((8192, 4096), dtype=torch.bfloat16, device=getitem_641.device)\n",
         "    out = torch.empty((S, H * D), dtype=torch.bfloat16, device=getitem_641.device)\n"),
    ],
    "v7/5c65f62b0422": [
        ("    S = 8192\n", "    S = getitem_642.shape[2]\n"),
    ],
    "v8/7884328a5557": [
        ("    M = 8192\n    N = 4096\n",
         "    N = _unsafe_view_981.numel()\n    M = mm_220.numel() // N\n"),
    ],
    "v7/7f544ceb2120": [
        ("    M = 8192\n    N = 4096\n",
         "    N = _unsafe_view_428.numel()\n    M = add_recomputed.numel() // N\n"),
        ("    BLOCK_N = 4096\n", "    BLOCK_N = triton.next_power_of_2(N)\n"),
    ],
    "v8/f4e9e58fef73": [],
    "v7/45990c83cfd6": [],
    "v7/1e49beb8a123": [],
    "v7/a12a160cb11b": [],
}

# benchmark configuration -> the reference problems whose kernels it times
CONFIG_PROBLEMS = {
    "C0F": ["v8/f4e9e58fef73"],
    "C1B": ["v7/45990c83cfd6"],
    "C2F": ["v7/1e49beb8a123"],
    "C2B": ["v7/a12a160cb11b"],
    "C3F": ["v8/c8c60d8f7015"],
    "C3B": ["v7/bfe872e373e4", "v7/5c65f62b0422"],
    "C4F": ["v8/7884328a5557"],
    "C4B": ["v7/7f544ceb2120"],
}


def _module_path(problem: str) -> Path:
    return OUT_DIR / (problem.replace("/", "_") + ".py")


def fetch(reference_root: str | Path) -> list[Path]:
    """Copy and patch the kernels from a reference checkout.  Returns the
    written files; raises if a file or a patch's original text is missing."""
    root = Path(reference_root)
    OUT_DIR.mkdir(parents=True, exist_ok=True)
    written, manifest = [], {}
    for problem, patches in PATCHES.items():
        src = root / problem / "optimized_kernel.py"
        text = src.read_text()
        sha_in = hashlib.sha256(text.encode()).hexdigest()
        for old, new in patches:
            n = text.count(old)
            if n != 1:
                raise RuntimeError(f"{problem}: patch target found {n} times: {old!r}")
            text = text.replace(old, new)
        dst = _module_path(problem)
        dst.write_text(text)
        written.append(dst)
        manifest[problem] = {"source_sha256": sha_in, "patches": len(patches)}
    (OUT_DIR / "manifest.json").write_text(json.dumps(manifest, indent=1))
    return written


def available() -> bool:
    return all(_module_path(p).exists() for p in PATCHES)


_cache: dict[str, object] = {}


def kernel_function(problem: str):
    """The reference's kernel_function for `problem` (fetched copy)."""
    fn = _cache.get(problem)
    if fn is None:
        path = _module_path(problem)
        if not path.exists():
            raise FileNotFoundError(f"{path} is missing: run oracle/triton_ref.py --reference <checkout>")
        spec = importlib.util.spec_from_file_location("triton_ref_" + problem.replace("/", "_"), path)
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        fn = _cache[problem] = mod.kernel_function
    return fn


if __name__ == "__main__":
    import argparse

    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--reference", required=True, help="path of a SherlockNoMad/KernelProblems checkout")
    a = ap.parse_args()
    for p in fetch(a.reference):
        print(p)
