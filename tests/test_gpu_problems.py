"""GPU parity of every drop-in kernel_function on the golden inputs.

For each reference problem: the drop-in (libfrag.so through the C ABI) runs on
the seeded golden inputs rebuilt on the GPU (same shapes and strides as the
reference's get_inputs), and must match
  * the output structure of the reference Model (count, shapes, dtypes, and
    which outputs are views of one buffer),
  * the pinned CPU oracle within the parity tolerances
    (bf16 atol 1e-2 / rtol 1.6e-2, fp32 rstd rtol 1e-4, embedding bit exact),
  * the golden rows the reference itself produced,
and fp32 reductions (dweight, table gradient) must match a float64 sum within
rtol 1e-4 (the reference graphs round those sums to bf16, see oracle)."""
import sys
from pathlib import Path

import pytest
import torch

from conftest import ORACLE_PREFIX as PREFIX
from conftest import assert_bf16_close, assert_bf16_sum_close, assert_f32_close
from kernelproblems_b200.problems import PROBLEMS
from oracle import fragments as F
from oracle.problems import ORACLES

GOLDEN = Path(__file__).resolve().parent / "golden"
sys.path.insert(0, str(GOLDEN))
from inputs import make_inputs  # noqa: E402

pytestmark = pytest.mark.gpu
FIXTURES = sorted(GOLDEN.glob("v*_*.pt"))

EXACT = {f"v{i}/1e49beb8a123" for i in range(1, 8)} | {  # gathers, and bf16 <-> fp32 casts
    f"v{i}/{h}" for i in range(1, 4) for h in ("dcf660c50ef3", "5d51b24b8d83", "b3f1b1135abc",
                                                "d800447a68f6", "3e3eb10963d7", "db48e1361360",
                                                "b508c9141fed")}
RMS_BWD = {"v7/45990c83cfd6", "v7/7f544ceb2120", "v8/d8f596b3df34", "v7/ed20955ec34b",
           "v8/43f0c930291e"}
EMB_BWD = {"v7/a12a160cb11b"}
# outputs that are copies out of an FSDP all-gather buffer (bit exact)
UNSHARD = {**{k: {1} for k in ("v8/8e33a91b7364", "v7/8e33a91b7364", "v6/8e33a91b7364",
                               "v5/013a3088b488", *(f"v{i}/18b859c50de2" for i in range(1, 5)))},
           "v8/94985bdb7630": set(range(3, 10)), "v8/7815074de963": set(range(3, 10)),
           "v8/12545c1e9b06": set(range(3, 9)),
           **{f"v{i}/2a844503364a": {2, 3, 4} for i in range(1, 5)},
           # the v-gradient passes through as a view of its input
           "v4/a1318bc813d2": {2}, "v5/a1bb72d946b0": {2}}
# norm -> embedding backward chain: output index of (dweight, table gradient)
CHAIN = {"v6/0b493aad68f0": (3, 4), "v5/118d525f44e0": (3, 4), "v4/680e4c57cdc8": (3, 4),
         "v3/680e4c57cdc8": (3, 4), "v2/680e4c57cdc8": (3, 4), "v1/680e4c57cdc8": (3, 4),
         "v8/f6251e84e3fa": (0, 1)}


def _chain_f64(key, cpu_in):
    """float64 dweight and table gradient of the norm -> embedding backward
    chain, from the oracle's bf16 dy and d_emb."""
    if key == "v6/0b493aad68f0":
        emb, w, mm_670, mm_672, mm_674, add_220, ids = cpu_in
    elif key == "v8/f6251e84e3fa":
        rec, mm_670, mm_672, mm_674, emb, w, add_220, ids = cpu_in
    else:
        g791, emb, mm_670, mm_672, mm_674, add_220, ids = cpu_in
        w = g791.contiguous().view(-1)
    rstd = rec[1] if key == "v8/f6251e84e3fa" else F.rmsnorm_fwd(emb, w, 1e-5)[1]
    v = [m.view(emb.shape) for m in (mm_670, mm_672, mm_674)]
    _, _, d_emb, dy = F.rmsnorm_embedding_bwd(emb, w, v, rstd, add_220, ids, 128256)
    return F.rmsnorm_dw_f64(dy, emb, rstd), F.embedding_bwd_f64(d_emb, ids, 128256), ids


# RMSNorm forward recomputed in its backward (frag_rmsnorm_fwd_bwd): variant
# of each snapshot; the dweight is the last output
FWD_BWD = {"v6/822931829090": "A3", "v5/92ce4a0c7b2c": "A3w",
           **{f"v{i}/363b7b58c971": "A3w" for i in range(1, 5)},
           "v6/e9198b707240": "A2", "v5/401b52261ef5": "A2w",
           **{f"v{i}/84c0a03c4374": "A2w" for i in range(1, 5)},
           "v6/408ac0979ac5": "B", "v5/cbfdd7549926": "Bw",
           **{f"v{i}/9c745ea697a7": "Bw" for i in range(1, 5)},
           "v6/28b45679fca1": "C", "v5/ac7d64b3c769": "C",
           **{f"v{i}/f7ad66842c19": "C" for i in range(1, 5)},
           "v8/3c6c589cdf81": "D"}


def _fwd_bwd_f64(key, cpu_in):
    """float64 dweight of the recompute-forward-in-backward problems, at the
    reference's own rstd of the bf16 normalised input h."""
    add = torch.ops.aten.add.Tensor
    sh = (1, 8192, 4096)
    kind = FWD_BWD[key]
    if kind in ("A3", "A3w", "A2", "A2w"):
        if kind.endswith("w"):
            g, h, *rest = cpu_in
            w = g.contiguous().view(-1)
        else:
            h, w, *rest = cpu_in
        mms = rest[:-1]
        dy = mms[0].view(sh)
        for m in mms[1:]:
            dy = add(dy, m.view(sh))
    elif kind in ("B", "Bw"):
        mm_3, emb, w, mm_a, mm_b, _ = cpu_in
        w = w.contiguous().view(-1)
        h = add(emb, mm_3.view(sh))
        dy = add(mm_a.view(sh), mm_b.view(sh))
    elif kind == "C":
        mm_223, x, mm_226, w = cpu_in
        h, dy = add(x, mm_223.view(sh)), mm_226.view(sh)
    else:
        mm_220, add_61, mm_223, mm_226, w = cpu_in
        h, dy = add(add(add_61, mm_220.view(sh)), mm_223.view(sh)), mm_226.view(sh)
    _, rstd = F.rmsnorm_fwd(h, w, 1e-5)
    return F.rmsnorm_dw_f64(dy, h, rstd)


def _check_structure(outs, fx):
    assert len(outs) == len(fx["outputs"]), "number of outputs"
    ptrs = [o.untyped_storage().data_ptr() for o in outs]
    for i, (o, ref) in enumerate(zip(outs, fx["outputs"])):
        assert list(o.shape) == ref["shape"], f"output {i} shape {list(o.shape)} != {ref['shape']}"
        assert str(o.dtype).split(".")[-1] == ref["dtype"], f"output {i} dtype"
        assert o.is_cuda
        assert ptrs.index(ptrs[i]) == ref["data_ptr_group"], f"output {i} aliasing differs"


def _dw_f64(key, cpu_in):
    if key == "v7/45990c83cfd6":
        x, w, dy = cpu_in
        _, rstd = F.rmsnorm_fwd(x, w, 1e-5)
        return F.rmsnorm_dw_f64(dy, x, rstd), (dy, x, rstd)
    if key == "v8/43f0c930291e":
        rec, mm_656, mm_658, mm_660, h, w, _ = cpu_in
        dy = torch.ops.aten.add.Tensor(mm_656.view(h.shape), mm_658.view(h.shape))
        dy = torch.ops.aten.add.Tensor(dy, mm_660.view(h.shape))
        return F.rmsnorm_dw_f64(dy, h, rec[1]), (dy, h, rec[1])
    if key == "v7/ed20955ec34b":
        mm_672, view_1794, mm_674, h, rstd, w, _ = cpu_in
        dy = torch.ops.aten.add.Tensor(view_1794, mm_672.view(h.shape))
        dy = torch.ops.aten.add.Tensor(dy, mm_674.view(h.shape))
        return F.rmsnorm_dw_f64(dy, h, rstd), (dy, h, rstd)
    if key == "v7/7f544ceb2120":
        mm_666, view_1776, h, rstd, w, _ = cpu_in
        dy = torch.ops.aten.add.Tensor(view_1776, mm_666.view(h.shape))
    else:
        mm_664, mm_666, h, rstd, w, _ = cpu_in
        dy = torch.ops.aten.add.Tensor(mm_664.view(h.shape), mm_666.view(h.shape))
    return F.rmsnorm_dw_f64(dy, h, rstd), (dy, h, rstd)


@pytest.mark.parametrize("fixture", FIXTURES, ids=lambda p: p.stem)
def test_problem_drop_in(fixture):
    fx = torch.load(fixture, weights_only=False)
    key = fx["problem"]
    # the oracle runs on the first input groups of PREFIX problems (the same
    # ops as the rest); every output is still checked against its golden rows
    ni, no = PREFIX.get(key.split("/")[1], (len(fx["inputs"]), len(fx["outputs"])))
    cpu_in = make_inputs(fx["inputs"][:ni])
    gpu_in = make_inputs(fx["inputs"], device="cuda")
    outs = PROBLEMS[key](*gpu_in)
    outs = outs if isinstance(outs, (tuple, list)) else (outs,)
    torch.cuda.synchronize()
    _check_structure(outs, fx)
    ref = ORACLES[key](*cpu_in)
    ref = ref if isinstance(ref, (tuple, list)) else (ref,)
    assert len(ref) == no
    ref = tuple(ref) + (None,) * (len(outs) - no)
    for i, (o, e, g) in enumerate(zip(outs, ref, fx["outputs"])):
        oc = o.cpu()
        rows = torch.tensor(g["rows"])
        o2 = oc.reshape(-1, oc.shape[-1]) if oc.dim() > 1 else oc.reshape(1, -1)
        # golden rows wider than the fixture's column cap are stored truncated
        o2 = o2[:, :g["cols"]] if "cols" in g else o2
        if e is None:  # beyond the oracle's prefix: the reference's golden rows
            assert o.dtype == torch.complex64
            assert_f32_close(torch.view_as_real(o2[rows]), torch.view_as_real(g["values"]),
                             f"output {i} golden rows", rtol=1e-5, atol=1e-5)
        elif key in EXACT:
            assert torch.equal(oc, e), "gathers and casts must be bit exact"
            assert torch.equal(o2[rows], g["values"]), "golden rows"
        elif i in UNSHARD.get(key, ()):
            assert torch.equal(oc, e), "unsharded parameter must be bit exact"
            assert torch.equal(o2[rows], g["values"]), "golden rows"
        elif key in EMB_BWD:
            ids = cpu_in[1]
            f64 = F.embedding_bwd_f64(cpu_in[0], ids, 128256)
            cnt = torch.bincount(ids.reshape(-1), minlength=128256).double()
            assert_f32_close(oc, f64, "table gradient vs float64", atol=(1e-4 * cnt.sqrt()).unsqueeze(1))
            untouched = cnt == 0
            assert torch.count_nonzero(oc[untouched]) == 0
        elif key in CHAIN and i == CHAIN[key][0]:
            dw64, _, _ = _chain_f64(key, cpu_in)
            assert_bf16_close(oc, e, "dweight vs the reference graph", atol=5e-2)
            assert_f32_close(oc, dw64, "dweight vs float64", atol=1e-3)
        elif key in CHAIN and i == CHAIN[key][1]:
            _, g64, ids = _chain_f64(key, cpu_in)
            cnt = torch.bincount(ids.reshape(-1), minlength=128256)
            # d_emb is a bf16 tensor in the graph: a rare one-ulp difference in
            # it (from a different fp32 summation order of the row reduction)
            # moves a table row by up to one bf16 ulp of |d_emb| (~0.06), the
            # reference harness's "reduction" tier (atol 0.125)
            assert_f32_close(oc, g64, "table gradient vs float64", atol=0.125)
            assert torch.count_nonzero(oc[cnt == 0]) == 0
            # No golden-row check here: the reference's CPU run accumulates
            # embedding_dense_backward in bf16 (torch 2.11's CPU kernel), so
            # with ~80 tokens per id its rows drift from the exact sum by
            # units; the CUDA aten kernel, like this one, sums in fp32.  The
            # oracle reproduces that CPU run bit for bit (test_oracle_golden),
            # and the float64 check above is the accuracy bar.
        elif key in FWD_BWD and FWD_BWD[key] != "C" and FWD_BWD[key] != "D" and i == len(outs) - 2:
            # dres + bf16(dx): the last input is dres
            assert_bf16_sum_close(oc, e, cpu_in[-1], "dres + dx")
            dres_rows = cpu_in[-1].reshape(-1, oc.shape[-1])[rows][:, :o2.shape[1]]
            assert_bf16_sum_close(o2[rows], g["values"], dres_rows, "dres + dx golden rows")
        elif key in FWD_BWD and i == len(outs) - 1:
            assert_bf16_close(oc.float(), e.float(), "dweight vs the reference graph", atol=5e-2)
            assert_f32_close(oc, _fwd_bwd_f64(key, cpu_in), "dweight vs float64", atol=1e-3)
        elif key in RMS_BWD and i == 1:
            f64, _ = _dw_f64(key, cpu_in)
            assert_bf16_close(oc.float(), e.float(), "dweight vs the reference graph", atol=5e-2)
            if oc.dtype == torch.float32:
                assert_f32_close(oc, f64, "dweight vs float64", atol=1e-3)
        elif key == "v7/0f38bc55457c" and i == 0:
            # fp32 q of a complex multiply: the same fp32 products, possibly
            # contracted into FMAs, so a few ulps of the products' magnitude
            assert_f32_close(oc, e, "q (fp32)", rtol=1e-5, atol=1e-5)
            assert_f32_close(o2[rows], g["values"], "q golden rows", rtol=1e-5, atol=1e-5)
        elif o.dtype == torch.complex64:
            # complex64 products, fp32 throughout: a few ulps (FMA contraction)
            assert_f32_close(torch.view_as_real(oc), torch.view_as_real(e), f"output {i} (complex64)",
                             rtol=1e-5, atol=1e-5)
            assert_f32_close(torch.view_as_real(o2[rows]), torch.view_as_real(g["values"]),
                             f"output {i} golden rows", rtol=1e-5, atol=1e-5)
        elif o.dtype == torch.float32:  # saved rstd
            assert_f32_close(oc, e, f"output {i} (fp32)")
            assert_f32_close(o2[rows], g["values"], f"output {i} golden rows")
        else:
            assert_bf16_close(oc, e, f"output {i}")
            assert_bf16_close(o2[rows], g["values"], f"output {i} golden rows")
