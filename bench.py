#!/usr/bin/env python
"""Fragment-suite benchmark: achieved HBM GB/s and tokens/s on B200.

One step = one pass of every hot-path fragment over its configuration's
synthetic batch, in this order (each fragment's inputs were last touched a
whole step — more than 17 GB of traffic — earlier, so every read is cold in
the 126 MB L2 without an explicit flush):

  C0F  RMSNorm fwd            x[4,2048,4096]
  C2F  embedding fwd          ids[8,4096] over table[128256,4096]
  C1B  RMSNorm bwd            x, grad[4,2048,4096]  (+ dweight exchange at N>1)
  C3F  RoPE fwd (neox)        q[8,4096,32,128], k[8,4096,8,128]
  C2B  embedding bwd          fp32 table gradient [128256,4096]
  C3B  RoPE bwd               grad_q, grad_k
  C4F  residual add + RMSNorm res, x[16,8192,8192]
  C4B  its backward           dy, dh, h -> d_res, dweight (+ exchange at N>1)

`value` = algorithmic bytes of the step on all ranks / max-over-ranks device
time per step (CUDA events on the launching stream, CUDA graphs).  At N>1
every rank runs its own batch (weak scaling); the only collective in the
step is the dweight exchange of C1B and C4B, which runs on its own stream
beside the fragments that follow it (C4B's beside the next step's first
fragments; the per-fragment breakdown times it inline instead).  By default
it is one single-CTA launch over NVLink peer memory (frag_dw_exchange_peer);
`--exchange nccl` uses the NCCL all-gather + fixed-order sum, which e2e
always uses (the two give the same bits).

After the timed steps, with the suite's results, the line carries:
  parity            each rank's dweight (C1B, C4B) against the float64 column
                    sum over all ranks' rows, and bit for bit against the
                    rank-order sum of separately gathered per-rank vectors;
  strong_scaling    C0F, C1B, C4F, C4B with the configured rows split over
                    the ranks (one global problem), kernel and exchange ms
                    apart, efficiency against each rank's own 1-GPU time;
  emb_vp            the vocab-parallel embedding (masked gather + NCCL
                    all-reduce of the output, per-rank gradient shard), with
                    gather / all-reduce / backward ms and bit-exact parity;
  triton_reference  (1 GPU) the reference's own Triton drop-ins beside this
                    library's drop-ins for the same problems, same inputs;
  e2e, cpu_baseline as the contract describes.

`--impl reference` times the reference's torch-eager CPU graph (restated in
oracle/fragments.py) on a row sample of the same workload on the host cores.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

METRIC = "achieved HBM GB/s (% of 8 TB/s) and tokens/s per fragment at 1/2/4/8 B200"
UNIT = "GB/s"
NOMINAL_HBM_GBS = 8000.0
FALLBACK_HBM_GBS = 6650.0
SUITE = ["C0F", "C2F", "C1B", "C3F", "C2B", "C3B", "C4F", "C4B"]
DOMINANT = "C4B"  # largest share of the step; its main kernel is the roofline kernel
# Fusions and callers beyond the five configurations, measured on request:
#   C2N  embedding gather + RMSNorm fused (C2 ids/table, eps 1e-5)
#   C3S  RoPE fwd writing q/k in the [B, H, S, D] layout attention reads (C3 shapes)
#   C2C  RMSNorm bwd -> embedding bwd chain fused (C2U: the same unfused)
#   C2S  FSDP table unshard + add/RMSNorm (one grouped copy, then the norm)
#   C2L  FSDP decoder-layer unshard (8 splits) + add/RMSNorm
#   C1R  RMSNorm forward recomputed in its backward, one pass (C1U: two calls)
#   C3X  complex64 RoPE of the v1/v2 snapshots (fp32 in and out)
NEXT = ["C2N", "C3S", "C2C", "C2U", "C2S", "C2L", "C1R", "C1U", "C3X"]


# ------------------------------------------------------------------ helpers

def parse_args(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=400)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default="suite",
                    help="suite | next | emb_vp | one fragment of " + ",".join(SUITE + NEXT))
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--exchange", choices=["peer", "nccl"], default="peer",
                    help="dweight exchange of C1B and C4B at N>1 in the timed steps: one launch over "
                         "NVLink peer memory (default), or NCCL all-gather + fixed-order sum")
    ap.add_argument("--no-extra", action="store_true",
                    help="skip the strong-scaling, vocab-parallel and Triton-reference legs")
    ap.add_argument("--e2e-steps", type=int, default=5)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=20.0,
                    help="target CPU time of the cpu_baseline sample")
    ap.add_argument("--ref-seconds", type=float, default=150.0,
                    help="target wall time of the whole --impl reference run")
    ap.add_argument("--no-clocks", action="store_true")
    ap.add_argument("--no-graphs", action="store_true", help="launch eagerly instead of graph replay")
    ap.add_argument("--rows-frac", type=float, default=1.0,
                    help="scale every config's rows/tokens (profiling captures of a smaller case only)")
    ap.add_argument("--json-out", default=None)
    return ap.parse_args(argv)


def env_rank():
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("LOCAL_RANK", "0")),
            int(os.environ.get("WORLD_SIZE", "1")))


def measured_peak():
    p = ROOT / "MEASURED_PEAKS.json"
    try:
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs: STREAM-style copy)"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback 6.65 TB/s (earlier measurement on this pool)"


def profile_traffic():
    """DRAM bytes per launch of the roofline kernel from the committed ncu summary."""
    p = ROOT / "profiles" / "roofline_traffic.json"
    try:
        d = json.loads(p.read_text())
        return d
    except Exception:
        return None


class ClockSampler:
    """SM clock, power and clock-event (throttle) reasons sampled during the
    timed region, read-only.  NVML is polled from a thread every `period_s`
    (5 ms), so even a timed region of a few tens of milliseconds carries a
    dozen samples; nvidia-smi at 100 ms is the fallback when NVML is not
    importable."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    # NVML clock-event reason bits (nvmlClocksEventReason*)
    BITS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20,
            "hw_thermal_slowdown": 0x40, "hw_power_brake_slowdown": 0x80}

    def __init__(self, device: torch.device, enabled: bool = True, period_s: float = 0.005):
        import threading
        self.rows, self.t0, self.t1 = [], None, None
        self.source = None
        self.proc = self.thread = None
        self.stop_ev = threading.Event()
        if not enabled:
            return
        try:
            import pynvml
            pynvml.nvmlInit()
            try:
                h = pynvml.nvmlDeviceGetHandleByUUID(
                    "GPU-" + str(torch.cuda.get_device_properties(device).uuid))
            except Exception:
                h = pynvml.nvmlDeviceGetHandleByIndex(device.index or 0)
            get_reasons = getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                pynvml.nvmlDeviceGetCurrentClocksThrottleReasons
            smax = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)

            def poll():
                while not self.stop_ev.is_set():
                    try:
                        self.rows.append(dict(
                            t=time.monotonic(), sm=float(pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)),
                            smax=float(smax), power=pynvml.nvmlDeviceGetPowerUsage(h) / 1000.0,
                            reasons=int(get_reasons(h))))
                    except Exception:
                        pass
                    self.stop_ev.wait(period_s)
            self.thread = threading.Thread(target=poll, daemon=True)
            self.thread.start()
            self.source = f"NVML every {period_s * 1e3:.0f} ms"
        except Exception:
            self._start_smi(device.index or 0)
        t_end = time.monotonic() + 5.0  # sampling runs before the timed region starts
        while not self.rows and time.monotonic() < t_end and self.source is not None:
            if self.proc is not None:
                self._read_smi()
            time.sleep(0.01)

    def _start_smi(self, idx):
        try:
            fd, self.path = tempfile.mkstemp(prefix="clocks_", suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-i", str(idx), "-lms", "100"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
            self.source = "nvidia-smi every 100 ms"
        except Exception:
            self.proc = None

    def _read_smi(self):
        rows = []
        for line in Path(self.path).read_text().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                bits = 0
                for name, col in (("hw_slowdown", 5), ("hw_thermal_slowdown", 6),
                                  ("sw_thermal_slowdown", 7), ("sw_power_cap", 8)):
                    if f[col].lower().startswith("active"):
                        bits |= self.BITS[name]
                rows.append(dict(t=None, sm=float(f[1]), smax=float(f[2]), power=float(f[3]),
                                 reasons=bits))
            except ValueError:
                continue
        self.rows = rows

    def start(self):
        """Mark the start of the timed region."""
        self.t0 = time.monotonic()
        self.n0 = len(self.rows)

    def stop(self):
        if self.source is None:
            return None
        self.t1 = time.monotonic()
        # one more sample after the region ends
        t_end = self.t1 + 1.0
        while len(self.rows) <= getattr(self, "n0", 0) and time.monotonic() < t_end:
            if self.proc is not None:
                self._read_smi()
            time.sleep(0.005)
        self.stop_ev.set()
        if self.thread is not None:
            self.thread.join(timeout=2)
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self._read_smi()
            os.unlink(self.path)
        n0 = getattr(self, "n0", 0)
        rows = [r for r in self.rows if r["t"] is None or self.t0 <= r["t"] <= self.t1] \
            if self.thread is not None else self.rows[max(0, n0 - 1):]
        if not rows:  # region shorter than one period: the samples around it
            rows = self.rows[max(0, n0 - 1): n0 + 1]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0,
                    "source": self.source}
        pmax = max(r["power"] for r in rows)
        load = [r for r in rows if r["power"] >= 0.5 * pmax] or rows
        reasons = sorted({name for r in rows for name, bit in self.BITS.items() if r["reasons"] & bit})
        return {"sm_mhz": statistics.median(r["sm"] for r in load),
                "sm_max_mhz": max(r["smax"] for r in rows),
                "sm_mhz_min": min(r["sm"] for r in rows),
                "reasons": reasons, "samples": len(rows),
                "power_w_max": pmax, "source": self.source}


def count_kernel_nodes(graph) -> int:
    """Kernel nodes in a captured torch CUDA graph (our launches incl. CUB's)."""
    try:
        from cuda.bindings import driver as cu
        g = cu.CUgraph(graph.raw_cuda_graph())
        err, _, n = cu.cuGraphGetNodes(g, 0)
        err, nodes, n = cu.cuGraphGetNodes(g, n)
        k = 0
        for nd in nodes[:n]:
            err, t = cu.cuGraphNodeGetType(nd)
            if t == cu.CUgraphNodeType.CU_GRAPH_NODE_TYPE_KERNEL:
                k += 1
        return k
    except Exception:
        return -1


# --------------------------------------------------------------- fragments

class Frag:
    """One fragment at its configuration on this rank: device-resident inputs,
    preallocated outputs, and the list of launch stages."""

    def __init__(self, name, desc, tokens, nbytes, stages, exchange=None, e2e=None):
        self.name, self.desc, self.tokens, self.bytes = name, desc, tokens, nbytes
        self.stages = stages          # [(label, callable)] local launches
        self.exchange = exchange      # callable or None (NCCL, run eagerly)
        self.e2e = e2e                # callable(host buffers) -> (h2d, d2h) via the public API
        self.kernel_nodes = 0
        self.ev = []                  # timing events: start, after each stage
        self.ev_end = None            # after the exchange (eager)


class Step:
    """The suite step.  Fragments are captured into CUDA graphs, one graph per
    run of fragments between NCCL exchanges (the whole step at N=1).  Two
    graph sets are captured: a plain one, replayed in the timed region, and an
    instrumented one with timing events recorded between fragments and stages
    (external event nodes), replayed only for the per-fragment breakdown."""

    def __init__(self, frags, use_graphs: bool):
        self.frags = frags
        self.comm = None  # stream of the overlapped exchanges (N > 1)
        for f in frags:  # warm: load kernels, size workspaces, first launches
            for _, fn in f.stages:
                fn()
        torch.cuda.synchronize()
        segs, cur = [], []
        for f in frags:
            cur.append(f)
            if f.exchange is not None:
                segs.append(cur)
                cur = []
        if cur:
            segs.append(cur)
        self.use_graphs = use_graphs
        self.plain, self.timed = [], []
        n_nodes = 0
        for seg in segs:
            for f in seg:
                f.ev = [torch.cuda.Event(enable_timing=True, external=use_graphs)
                        for _ in range(len(f.stages) + 1)]
                f.ev_end = torch.cuda.Event(enable_timing=True) if f.exchange is not None else None
            gp = gt = None
            if use_graphs:
                gp = torch.cuda.CUDAGraph(keep_graph=True)
                with torch.cuda.graph(gp, capture_error_mode="thread_local"):
                    self._launch(seg, events=False)
                n_nodes += max(count_kernel_nodes(gp), 0)
                gp.instantiate()
                gt = torch.cuda.CUDAGraph()
                with torch.cuda.graph(gt, capture_error_mode="thread_local"):
                    self._launch(seg, events=True)
            self.plain.append((gp, seg))
            self.timed.append((gt, seg))
        torch.cuda.synchronize()
        self.kernel_nodes = n_nodes if use_graphs else None

    @staticmethod
    def _launch(seg, events):
        for f in seg:
            if events:
                f.ev[0].record()
            for si, (_, fn) in enumerate(f.stages):
                fn()
                if events:
                    f.ev[si + 1].record()

    def _run(self, graphs, events):
        main = torch.cuda.current_stream()
        overlap = not events and any(seg[-1].exchange is not None for _, seg in graphs)
        if overlap and self.comm is None:
            self.comm = torch.cuda.Stream()
        if not hasattr(self, "ex_done"):
            self.ex_done = [None] * len(graphs)
        for si, (g, seg) in enumerate(graphs):
            if overlap and self.ex_done[si] is not None:
                # the previous step's exchange of this segment reads the
                # dweight this segment is about to rewrite: order after it
                # (it finished long ago in practice: a whole step runs between)
                main.wait_event(self.ex_done[si])
            if g is not None:
                g.replay()
            else:
                self._launch(seg, events)
            last = seg[-1]
            if last.exchange is not None:
                if overlap:
                    # The exchange (dweight all-gather + fixed-order sum) runs
                    # on its own stream after this segment's kernels, beside
                    # the fragments that follow -- for the last segment, beside
                    # the next step's first fragments -- none of which reads
                    # its result.
                    done = torch.cuda.Event()
                    done.record(main)
                    self.comm.wait_event(done)
                    with torch.cuda.stream(self.comm):
                        last.exchange()
                    ev = torch.cuda.Event()
                    ev.record(self.comm)
                    self.ex_done[si] = ev
                else:
                    last.exchange()
                if events:
                    last.ev_end.record()

    def join(self):
        """Order the current stream after every exchange still in flight."""
        if self.comm is not None:
            torch.cuda.current_stream().wait_stream(self.comm)

    def run(self):
        """One step as timed: no timing events inside; NCCL exchanges overlap
        the fragments that follow them (call join() before reading results)."""
        self._run(self.plain, events=False)

    def run_instrumented(self):
        self.join()
        self._run(self.timed, events=True)

    def release(self):
        self.plain, self.timed = [], []

    def breakdown(self):
        """Per-fragment and per-stage ms of the last instrumented step."""
        out = {}
        for f in self.frags:
            st = [f.ev[i].elapsed_time(f.ev[i + 1]) for i in range(len(f.stages))]
            end = f.ev_end if f.ev_end is not None else f.ev[-1]
            out[f.name] = (f.ev[0].elapsed_time(end), st)
        return out


def scaled_configs(frac: float):
    """The five configs with their row (token) dimension scaled by frac."""
    from dataclasses import replace

    from kernelproblems_b200 import configs as cf
    if frac == 1.0:
        return cf.C0, cf.C1, cf.C2, cf.C3, cf.C4

    def rows(cfg):
        m = max(1, int(round(cfg.M * frac)))
        return replace(cfg, shape=(m, cfg.N))
    c2 = replace(cf.C2, batch=(1, max(1, int(round(cf.C2.T * frac)))))
    c3 = replace(cf.C3, B=max(1, int(round(cf.C3.B * frac))))
    return rows(cf.C0), rows(cf.C1), c2, c3, rows(cf.C4)


def build_suite(dev, world, rank, names, pg, frac=1.0, exchange="peer"):
    """Build the requested fragments.  Each builder has its own scope, so the
    launch closures never see another fragment's tensors."""
    from kernelproblems_b200 import configs as cf
    from kernelproblems_b200 import ops
    seed0 = 1000 * rank
    C0, C1, C2, C3, C4 = scaled_configs(frac)

    def exchange_dw(dw_part, dw_out, parts_buf):
        """(exchange the step uses, NCCL exchange, peer object or None).  The
        NCCL exchange all-gathers the per-rank dweights and adds them in rank
        order; the peer exchange (one single-CTA launch over NVLink peer
        memory) gives the same bits.  Peer set-up is collective: it either
        works on every rank or raises on every rank, which then all keep
        NCCL."""
        if world == 1:
            return None, None, None

        def ex_nccl():
            dist.all_gather_into_tensor(parts_buf.view(-1), dw_part, group=pg)
            ops.dw_reduce(parts_buf, out=dw_out)
        if exchange != "peer":
            return ex_nccl, ex_nccl, None
        from kernelproblems_b200 import sharding
        try:
            peer = sharding.PeerDweightExchange(dw_part.numel(), group=pg, device=dev)
        except RuntimeError:
            return ex_nccl, ex_nccl, None

        def ex_peer():
            peer(dw_part, out=dw_out)
        return ex_peer, ex_nccl, peer

    def mk_c0f():
        c = C0
        x = cf.randn(c.shape, device=dev, seed=seed0 + 1)
        w = cf.rmsnorm_weight(c.N, device=dev, seed=seed0 + 2)
        y = torch.empty_like(x)
        r = torch.empty(c.shape[:-1], dtype=torch.float32, device=dev)
        f = Frag("C0F", c.name, c.M, cf.bytes_rmsnorm_fwd(c.M, c.N),
                 [("rmsnorm_fwd", lambda: ops.rmsnorm_fwd(x, w, c.eps, out=y, rstd=r))])
        f.host = dict(x=x)
        f.e2e = lambda h: _e2e_call(lambda xs: ops.rmsnorm_fwd(xs["x"], w, c.eps), h)
        return f

    def mk_rms_bwd(name, c, with_dres, s, split_stages):
        w = cf.rmsnorm_weight(c.N, device=dev, seed=seed0 + s)
        x = cf.randn(c.shape, device=dev, seed=seed0 + s + 1)
        g = cf.randn(c.shape, device=dev, seed=seed0 + s + 2)
        dh = cf.randn(c.shape, device=dev, seed=seed0 + s + 3) if with_dres else None
        _, r = ops.rmsnorm_fwd(x, w, c.eps)
        ws = torch.empty(ops.rmsnorm_bwd_workspace_bytes(c.M, c.N), dtype=torch.uint8, device=dev)
        G = ops.rmsnorm_bwd_num_blocks(c.M, c.N)
        parts = ws[: G * c.N * 4].view(torch.float32).view(G, c.N)
        dw = torch.empty(c.N, dtype=torch.float32, device=dev)
        dwg = torch.empty(c.N, dtype=torch.float32, device=dev)
        pbuf = torch.empty(world, c.N, dtype=torch.float32, device=dev)
        nb = cf.bytes_add_rmsnorm_bwd(c.M, c.N) if with_dres else cf.bytes_rmsnorm_bwd(c.M, c.N)
        ex, ex_nccl, peer = exchange_dw(dw, dwg, pbuf)
        if split_stages:
            # row kernel and dweight reduce as two timed stages (the row kernel
            # is the roofline kernel)
            stages = [("rmsnorm_bwd_main", lambda: ops.rmsnorm_bwd(g, x, r, w, dres=dh, dw_dtype=None,
                                                                  workspace=ws)),
                      ("dw_reduce", lambda: ops.dw_reduce(parts, out=dw))]
            f = Frag(name, c.name + (" bwd" if with_dres else ""), c.M, nb, stages, exchange=ex)
        else:
            # one call, as a user makes it: row kernel + dependent dweight
            # reduce, into fixed outputs (every captured graph writes the same
            # buffers the exchange and the parity check read)
            dx = torch.empty_like(x)
            f = Frag(name, c.name + (" bwd" if with_dres else ""), c.M, nb,
                     [("rmsnorm_bwd", lambda: ops.rmsnorm_bwd(g, x, r, w, dres=dh, workspace=ws,
                                                              dx_out=dx, dw_out=dw))],
                     exchange=ex)
        # e2e keeps the NCCL exchange: its steps are host-copy bound, and ranks
        # can drift further apart there than the peer kernel's bounded waits allow
        f.exchange_e2e = ex_nccl
        f.peer = peer
        f.exchange_kind = None if world == 1 else ("peer" if peer is not None else "nccl")
        f.host = dict(g=g, x=x, r=r) if dh is None else dict(g=g, x=x, r=r, dh=dh)
        f.e2e = lambda h: _e2e_call(lambda xs: ops.rmsnorm_bwd(xs["g"], xs["x"], xs["r"], w,
                                                               dres=xs.get("dh")), h)
        # for the dweight parity check: the terms, this rank's dweight, the
        # exchanged (global) dweight
        f.dw_check = dict(g=g, x=x, r=r, local=lambda: dw, glob=(lambda: dwg) if world > 1 else None)
        return f

    def mk_c2(which):
        c = C2
        ids = cf.embedding_ids(c, device=dev, seed=2 + rank)
        if which == "C2F":
            table = cf.randn((c.vocab, c.dim), std=0.02, device=dev, seed=seed0 + 7)
            out = torch.empty(*c.batch, c.dim, dtype=torch.bfloat16, device=dev)
            f = Frag("C2F", c.name + " fwd", c.T, cf.bytes_embedding_fwd(c.T, c.dim),
                     [("embedding_fwd", lambda: ops.embedding_fwd(ids, table, out=out))])
            f.host = dict(ids=ids)
            f.e2e = lambda h: _e2e_call(lambda xs: ops.embedding_fwd(xs["ids"], table), h)
            return f
        gr = cf.randn((*c.batch, c.dim), device=dev, seed=seed0 + 8)
        Gt = torch.empty(c.vocab, c.dim, dtype=torch.float32, device=dev)
        wsb = torch.empty(max(16, ops._lib.load().frag_embedding_bwd_workspace_bytes(c.T, c.vocab)),
                          dtype=torch.uint8, device=dev)
        f = Frag("C2B", c.name + " bwd", c.T, cf.bytes_embedding_bwd(c.T, c.dim, c.vocab),
                 [("embedding_bwd", lambda: ops.embedding_bwd(gr, ids, c.vocab, out=Gt, workspace=wsb))])
        f.host = dict(g=gr, ids=ids)
        f.e2e = lambda h: _e2e_call(lambda xs: ops.embedding_bwd(xs["g"], xs["ids"], c.vocab), h)
        return f

    def mk_c3(which):
        c = C3
        inv = which == "C3B"
        s = 13 if inv else 11
        pos = cf.rope_positions(c, device=dev)
        q = cf.randn((c.B, c.S, c.Hq, c.D), device=dev, seed=seed0 + s)
        k = cf.randn((c.B, c.S, c.Hk, c.D), device=dev, seed=seed0 + s + 1)
        oq, ok = torch.empty_like(q), torch.empty_like(k)
        f = Frag(which, c.name + (" bwd" if inv else " fwd"), c.T, cf.bytes_rope(c.T, c.Hq, c.Hk, c.D),
                 [("rope", lambda: ops.rope(q, k, pos, theta=c.theta, inverse=inv, out_q=oq, out_k=ok))])
        f.host = dict(q=q, k=k)
        f.e2e = lambda h: _e2e_call(lambda xs: ops.rope(xs["q"], xs["k"], pos, theta=c.theta,
                                                        inverse=inv), h)
        return f

    def mk_c3x():
        # the v1/v2 snapshots' RoPE: complex64 q [1, 8192, 32, 64] and
        # k [1, 8192, 8, 64] times freqs_cis[pos] (v2/075cb40f3d5d shapes)
        S, Hq, Hk, D2 = 8192, 32, 8, 64
        g = torch.Generator(device=dev).manual_seed(seed0 + 60)
        q = torch.randn((1, S, Hq, D2), dtype=torch.complex64, device=dev, generator=g)
        k = torch.randn((1, S, Hk, D2), dtype=torch.complex64, device=dev, generator=g)
        freqs = torch.randn((S, D2), dtype=torch.complex64, device=dev, generator=g)
        pos = torch.randint(0, S, (1, S), dtype=torch.int32, device=dev, generator=g)
        oq, ok = torch.empty_like(q), torch.empty_like(k)
        nb = 2 * S * (Hq + Hk) * D2 * 8 + S * 4 + S * D2 * 8
        f = Frag("C3X", "complex64 RoPE q[1,8192,32,64] k[1,8192,8,64] x freqs_cis[pos]", S, nb,
                 [("rope_complex", lambda: ops.rope_complex(q, k, pos, freqs, out_q=oq, out_k=ok))])
        f.host = dict(q=q, k=k)
        f.e2e = lambda h: _e2e_call(lambda xs: ops.rope_complex(xs["q"], xs["k"], pos, freqs), h)
        return f

    def mk_c4f():
        c = C4
        w = cf.rmsnorm_weight(c.N, device=dev, seed=seed0 + 20)
        res = cf.randn(c.shape, device=dev, seed=seed0 + 21)
        x = cf.randn(c.shape, device=dev, seed=seed0 + 22)
        h = torch.empty_like(x)
        y = torch.empty_like(x)
        f = Frag("C4F", c.name + " fwd", c.M, cf.bytes_add_rmsnorm_fwd(c.M, c.N),
                 [("add_rmsnorm_fwd", lambda: ops.add_rmsnorm_fwd(res, x, w, c.eps, h_out=h, y_out=y))])
        f.host = dict(res=res, x=x)
        f.e2e = lambda h_: _e2e_call(lambda xs: ops.add_rmsnorm_fwd(xs["res"], xs["x"], w, c.eps), h_)
        return f

    def mk_c2n():
        # embedding gather fused with RMSNorm (the first attention_norm), C2 shapes
        c = C2
        ids = cf.embedding_ids(c, device=dev, seed=2 + rank)
        table = cf.randn((c.vocab, c.dim), std=0.02, device=dev, seed=seed0 + 7)
        w = cf.rmsnorm_weight(c.dim, device=dev, seed=seed0 + 9)
        f = Frag("C2N", c.name + " fwd + RMSNorm fused", c.T,
                 cf.bytes_embedding_fwd(c.T, c.dim) + c.dim * cf.BF16,
                 [("embedding_rmsnorm_fwd", lambda: ops.embedding_rmsnorm_fwd(ids, table, w, 1e-5))])
        f.host = dict(ids=ids)
        f.e2e = lambda h: _e2e_call(lambda xs: ops.embedding_rmsnorm_fwd(xs["ids"], table, w, 1e-5)[0], h)
        return f

    def mk_c3s():
        # RoPE fwd writing the [B, H, S, D] layout attention reads, C3 shapes
        c = C3
        pos = cf.rope_positions(c, device=dev)
        q = cf.randn((c.B, c.S, c.Hq, c.D), device=dev, seed=seed0 + 15)
        k = cf.randn((c.B, c.S, c.Hk, c.D), device=dev, seed=seed0 + 16)
        oq = torch.empty((c.B, c.Hq, c.S, c.D), dtype=q.dtype, device=dev).transpose(1, 2)
        ok = torch.empty((c.B, c.Hk, c.S, c.D), dtype=k.dtype, device=dev).transpose(1, 2)
        f = Frag("C3S", c.name + " fwd into [B,H,S,D]", c.T, cf.bytes_rope(c.T, c.Hq, c.Hk, c.D),
                 [("rope_bhsd", lambda: ops.rope(q, k, pos, theta=c.theta, out_q=oq, out_k=ok))])
        f.host = dict(q=q, k=k)
        f.e2e = lambda h: _e2e_call(lambda xs: ops.rope(xs["q"], xs["k"], pos, theta=c.theta,
                                                        out_layout="bhsd"), h)
        return f

    def mk_chain(which):
        # RMSNorm backward -> residual add -> embedding backward at the shapes
        # of the reference chain problem (v6/0b493aad68f0: 8192 tokens, width
        # 4096, 128256-row table, ids uniform in [0, 100), three summed
        # gradients, rstd recomputed, y returned).  C2C is the fused kernel;
        # C2U the same chain composed of the unfused calls (d_emb round trip).
        T, D, V = 8192, 4096, 128256
        x = cf.randn((1, T, D), device=dev, seed=seed0 + 30)
        w = cf.randn((D,), device=dev, seed=seed0 + 31)
        dys = [cf.randn((T, D), device=dev, seed=seed0 + 32 + j) for j in range(3)]
        dres = cf.randn((1, T, D), device=dev, seed=seed0 + 35)
        gen = torch.Generator(device=dev)
        gen.manual_seed(seed0 + 36)
        ids = torch.randint(0, 100, (1, T), generator=gen, device=dev)
        Gt = torch.empty(V, D, dtype=torch.float32, device=dev)
        nb = cf.bytes_rmsnorm_embedding_bwd(T, D, V)
        name = "norm bwd -> embedding bwd chain [8192,4096] vocab 128256"
        if which == "C2C":
            ws = torch.empty(max(16, ops._lib.load().frag_rmsnorm_embedding_bwd_workspace_bytes(T, D, V)),
                             dtype=torch.uint8, device=dev)
            f = Frag("C2C", name + " fused", T, nb,
                     [("rmsnorm_embedding_bwd",
                       lambda: ops.rmsnorm_embedding_bwd(x, w, ids, dys, V, dres=dres, eps=1e-5,
                                                         write_y=True, out=Gt, workspace=ws))])
            f.host = dict(x=x, g0=dys[0], g1=dys[1], g2=dys[2], dres=dres, ids=ids)
            f.e2e = lambda h: _e2e_call(lambda xs: ops.rmsnorm_embedding_bwd(
                xs["x"], w, xs["ids"], [xs["g0"], xs["g1"], xs["g2"]], V, dres=xs["dres"], eps=1e-5,
                write_y=True), h)
            return f
        wsb = torch.empty(max(16, ops._lib.load().frag_embedding_bwd_workspace_bytes(T, V)),
                          dtype=torch.uint8, device=dev)
        y = torch.empty_like(x)
        r = torch.empty((1, T), dtype=torch.float32, device=dev)

        def unfused(x, g0, g1, g2, dres, ids, out=None, ws=None, y=None, r=None):
            y, r = ops.rmsnorm_fwd(x, w, 1e-5, out=y, rstd=r)
            dy01 = torch.add(g0, g1).view(x.shape)
            d_emb, dw = ops.rmsnorm_bwd(dy01, x, r, w, dy2=g2.view(x.shape), dres=dres)
            return ops.embedding_bwd(d_emb, ids, V, out=out, workspace=ws), dw, y
        f = Frag("C2U", name + " unfused", T, nb,
                 [("chain_unfused", lambda: unfused(x, *dys, dres, ids, out=Gt, ws=wsb, y=y, r=r))])
        f.host = dict(x=x, g0=dys[0], g1=dys[1], g2=dys[2], dres=dres, ids=ids)
        f.e2e = lambda h: _e2e_call(lambda xs: unfused(**xs), h)
        return f

    def mk_fwd_bwd(tag):
        # RMSNorm forward recomputed in its backward at the shapes of
        # v6/822931829090 (x [8192, 4096], dy = mm_656 + mm_658 + mm_660,
        # dres, y returned): one frag_rmsnorm_fwd_bwd pass (C1R), or the
        # forward and the backward as two calls (C1U)
        M, N = 8192, 4096
        w = cf.rmsnorm_weight(N, device=dev, seed=seed0 + 50)
        x = cf.randn((1, M, N), device=dev, seed=seed0 + 51)
        dys = [cf.randn((1, M, N), device=dev, seed=seed0 + 52 + i) for i in range(3)]
        dres = cf.randn((1, M, N), device=dev, seed=seed0 + 55)
        ws = torch.empty(ops.rmsnorm_bwd_workspace_bytes(M, N), dtype=torch.uint8, device=dev)

        def fused(x, d0, d1, d2, dres):
            return ops.rmsnorm_fwd_bwd(x, w, d0, dy2=d1, dy3=d2, dres=dres, eps=1e-5, workspace=ws)

        def unfused(x, d0, d1, d2, dres):
            y, r = ops.rmsnorm_fwd(x, w, 1e-5)
            dx, dw = ops.rmsnorm_bwd(d0, x, r, w, dy2=d1, dy3=d2, dres=dres, eps=1e-5, workspace=ws)
            return y, dx, dw
        fn = fused if tag == "C1R" else unfused
        label = ("RMSNorm fwd recomputed in bwd [8192,4096], 3 grads + dres, "
                 + ("fused" if tag == "C1R" else "fwd then bwd"))
        f = Frag(tag, label, M, cf.bytes_rmsnorm_fwd_bwd(M, N, 1, 3, True, True),
                 [("rmsnorm_fwd_bwd" if tag == "C1R" else "rmsnorm_fwd+bwd",
                   lambda: fn(x, *dys, dres))])
        f.host = dict(x=x, d0=dys[0], d1=dys[1], d2=dys[2], dres=dres)
        f.e2e = lambda h: _e2e_call(lambda xs: fn(**xs), h)
        return f

    def mk_unshard(tag, splits, ncopy, label):
        # FSDP unshard of parameters out of one all-gather buffer viewed
        # [8, -1] (split 0 the norm weight) in one grouped copy, plus the add
        # + RMSNorm with the gathered weight, at the reference's shapes
        M, N, W = 8192, 4096, 8
        res = cf.randn((1, M, N), device=dev, seed=seed0 + 40)
        x = cf.randn((M, N), device=dev, seed=seed0 + 41)
        flat = cf.randn((W * sum(splits),), device=dev, seed=seed0 + 42)
        outs = [torch.empty(W, n, dtype=torch.bfloat16, device=dev) for n in splits[:ncopy]]
        y = torch.empty_like(res)

        def step(res, x, flat, outs=None, y=None):
            parts = ops.copy_rows_grouped(torch.split(flat.view(W, -1), splits, dim=1)[:ncopy], outs)
            _, yy, _ = ops.add_rmsnorm_fwd(res, x.view(res.shape), parts[0].view(-1), 1e-5,
                                           write_h=False, save_rstd=False, y_out=y)
            return yy, parts
        f = Frag(tag, label, M, cf.bytes_add_rmsnorm_unshard(M, N, W, sum(splits[1:ncopy])),
                 [("unshard_add_rmsnorm", lambda: step(res, x, flat, outs=outs, y=y))])
        f.host = dict(res=res, x=x, flat=flat)
        f.e2e = lambda h: _e2e_call(lambda xs: step(xs["res"], xs["x"], xs["flat"]), h)
        return f

    def mk_c2s():
        # v8/8e33a91b7364: buffer [525340672], splits [512, 65667072]
        return mk_unshard("C2S", [512, 65667072], 2,
                          "FSDP table unshard + add/RMSNorm [8192,4096] (8 shards of 65667072)")

    def mk_c2l():
        # v8/7815074de963: one decoder layer's buffer [218112000], splits
        # [512, 2097152, 524288, 524288, 2097152, 512, 7340032 x3], 0-7 copied
        sp = [512, 2097152, 524288, 524288, 2097152, 512, 7340032, 7340032, 7340032]
        return mk_unshard("C2L", sp, 8,
                          "FSDP layer unshard (8 splits) + add/RMSNorm [8192,4096]")

    builders = {"C2N": mk_c2n, "C3S": mk_c3s, "C2S": mk_c2s, "C2L": mk_c2l,
                "C1R": lambda: mk_fwd_bwd("C1R"), "C3X": mk_c3x, "C1U": lambda: mk_fwd_bwd("C1U"), "C2C": lambda: mk_chain("C2C"),
                "C2U": lambda: mk_chain("C2U"), "C0F": mk_c0f, "C1B": lambda: mk_rms_bwd("C1B", C1, False, 3, False),
                "C2F": lambda: mk_c2("C2F"), "C2B": lambda: mk_c2("C2B"),
                "C3F": lambda: mk_c3("C3F"), "C3B": lambda: mk_c3("C3B"),
                "C4F": mk_c4f, "C4B": lambda: mk_rms_bwd("C4B", C4, True, 23, True)}
    return [builders[n]() for n in SUITE + NEXT if n in names]


# (h2d stream, d2h stream) while e2e_measure runs, else None
_E2E_PIPE = None


def _e2e_call(fn, host, pipe=None):
    """Copy `host` (pinned) inputs to the device, run the public API call, copy
    every output tensor back into pinned memory.  Returns (h2d, d2h) bytes.

    With `pipe` = (h2d stream, d2h stream) the uploads and read-backs run on
    their own streams, ordered by stream waits: the call waits for its own
    uploads, the read-back waits for the call.  Consecutive calls then overlap
    one call's read-back, the next call's kernels and the one after's upload
    (the copy engines work in both directions at once)."""
    dev = torch.device("cuda", torch.cuda.current_device())
    cur = torch.cuda.current_stream(dev)
    pipe = pipe if pipe is not None else _E2E_PIPE
    if pipe is None:
        xs = {k: v.to(dev, non_blocking=True) for k, v in host["in"].items()}
    else:
        h2d_s, d2h_s = pipe
        with torch.cuda.stream(h2d_s):
            xs = {k: v.to(dev, non_blocking=True) for k, v in host["in"].items()}
        cur.wait_stream(h2d_s)
        for t in xs.values():
            t.record_stream(cur)
    outs = fn(xs)
    outs = outs if isinstance(outs, (tuple, list)) else (outs,)
    h2d = sum(v.numel() * v.element_size() for v in host["in"].values())
    d2h = 0
    flat = [t for o in outs for t in (o if isinstance(o, (tuple, list)) else (o,))]
    tensors = [o for o in flat if isinstance(o, torch.Tensor)]
    if pipe is not None:
        d2h_s.wait_stream(cur)
    for i, o in enumerate(tensors):
        buf = host["out"].get(i)
        if buf is None or buf.shape != o.shape or buf.dtype != o.dtype:
            buf = torch.empty(o.shape, dtype=o.dtype, pin_memory=True)
            host["out"][i] = buf
        if pipe is None:
            buf.copy_(o, non_blocking=True)
        else:
            o.record_stream(d2h_s)
            with torch.cuda.stream(d2h_s):
                buf.copy_(o, non_blocking=True)
        d2h += o.numel() * o.element_size()
    return h2d, d2h


# ------------------------------------------------------------------ CPU arm

def cpu_suite_sample(frac: float, names):
    """Build the CPU sample: each fragment's config with rows (tokens) scaled
    by `frac` (embedding: tokens and vocab).  Returns [(name, bytes, tokens, fn)]."""
    from kernelproblems_b200 import configs as cf
    from oracle import fragments as ora
    out = []

    def rows(M):
        return max(1, int(round(M * frac)))
    if "C0F" in names:
        c = cf.C0
        m = rows(c.M)
        x = cf.randn((m, c.N), seed=1)
        w = cf.rmsnorm_weight(c.N)
        out.append(("C0F", cf.bytes_rmsnorm_fwd(m, c.N), m, lambda x=x, w=w, eps=c.eps: ora.rmsnorm_fwd(x, w, eps)))
    if "C2F" in names or "C2B" in names:
        c = cf.C2
        t = rows(c.T)
        V = max(1, int(round(c.vocab * frac)))
        cs = cf.EmbeddingCfg("sample", (1, t), V, c.dim)
        ids = cf.embedding_ids(cs).reshape(-1)
        if "C2F" in names:
            table = cf.randn((V, c.dim), std=0.02, seed=7)
            out.append(("C2F", cf.bytes_embedding_fwd(t, c.dim), t,
                        lambda ids=ids, table=table: ora.embedding_fwd(table, ids)))
        if "C2B" in names:
            g = cf.randn((t, c.dim), seed=8)
            out.append(("C2B", cf.bytes_embedding_bwd(t, c.dim, V), t,
                        lambda g=g, ids=ids, V=V: ora.embedding_bwd(g, ids, V)))
    if "C1B" in names:
        c = cf.C1
        m = rows(c.M)
        x = cf.randn((m, c.N), seed=3)
        w = cf.rmsnorm_weight(c.N)
        g = cf.randn((m, c.N), seed=5)
        _, r = ora.rmsnorm_fwd(x, w, c.eps)
        out.append(("C1B", cf.bytes_rmsnorm_bwd(m, c.N), m,
                    lambda g=g, x=x, r=r, w=w: ora.rmsnorm_bwd(g, x, r, w)))
    if "C3F" in names or "C3B" in names:
        c = cf.C3
        s = max(1, int(round(c.S * frac * c.B)))
        q = cf.randn((1, s, c.Hq, c.D), seed=11)
        k = cf.randn((1, s, c.Hk, c.D), seed=12)
        pos = torch.arange(s) % c.S
        for nm, inv in (("C3F", False), ("C3B", True)):
            if nm in names:
                out.append((nm, cf.bytes_rope(s, c.Hq, c.Hk, c.D), s,
                            lambda q=q, k=k, pos=pos, inv=inv, th=c.theta: (ora.rope_neox(q, pos, th, inv),
                                                                       ora.rope_neox(k, pos, th, inv))))
    if "C4F" in names or "C4B" in names:
        c = cf.C4
        m = rows(c.M)
        w = cf.rmsnorm_weight(c.N)
        res = cf.randn((m, c.N), seed=21)
        x = cf.randn((m, c.N), seed=22)
        if "C4F" in names:
            out.append(("C4F", cf.bytes_add_rmsnorm_fwd(m, c.N), m,
                        lambda res=res, x=x, w=w, eps=c.eps: ora.add_rmsnorm_fwd(res, x, w, eps)))
        if "C4B" in names:
            h, _, r = ora.add_rmsnorm_fwd(res, x, w, c.eps)
            dy = cf.randn((m, c.N), seed=24)
            out.append(("C4B", cf.bytes_add_rmsnorm_bwd(m, c.N), m,
                        lambda dy=dy, h=h, r=r, w=w, dh=x: ora.add_rmsnorm_bwd(dy, None, h, r, w, dh)))
    order = {n: i for i, n in enumerate(SUITE)}
    return sorted(out, key=lambda t: order[t[0]])


def run_cpu_sample(sample, reps: int = 1):
    t_tot, b_tot, per = 0.0, 0, {}
    for name, nb, tok, fn in sample:
        fn()  # warm
        t0 = time.perf_counter()
        for _ in range(reps):
            fn()
        dt = (time.perf_counter() - t0) / reps
        per[name] = {"s": dt, "GB/s": nb / dt / 1e9, "tokens/s": tok / dt}
        t_tot += dt
        b_tot += nb
    return b_tot / t_tot / 1e9, t_tot, per


def calibrate_cpu(names, target_s: float):
    """Pick a row fraction whose suite sample takes about target_s on the CPU."""
    torch.set_num_threads(os.cpu_count() or 1)
    f0 = 1.0 / 64
    _, t0, _ = run_cpu_sample(cpu_suite_sample(f0, names))
    f = min(1.0, max(1.0 / 4096, f0 * target_s / max(t0, 1e-6)))
    return f


def cpu_baseline(names, target_s: float):
    frac = calibrate_cpu(names, target_s / 2)
    sample = cpu_suite_sample(frac, names)
    gbs, t, per = run_cpu_sample(sample)
    return {"value": round(gbs, 3), "unit": UNIT, "cores": torch.get_num_threads(), "kind": "port",
            "sample": (f"torch-eager CPU restatement of the reference graphs (oracle/fragments.py), "
                       f"each fragment on {frac:.4g} of its config's rows (embedding: tokens and vocab), "
                       f"{t:.1f} s"),
            "fragments": {k: {"GB/s": round(v["GB/s"], 3)} for k, v in per.items()}}


# ---------------------------------------------------------------- main arms

def suite_descriptions(names, other: dict | None = None) -> dict:
    """Config name of each suite fragment (both arms report the same), the
    given description of any other."""
    from kernelproblems_b200 import configs as cf
    desc = {"C0F": cf.C0.name, "C1B": cf.C1.name, "C2F": cf.C2.name + " fwd",
            "C2B": cf.C2.name + " bwd fp32 table", "C3F": cf.C3.name + " fwd",
            "C3B": cf.C3.name + " bwd", "C4F": cf.C4.name + " fwd", "C4B": cf.C4.name + " bwd"}
    return {n: desc.get(n, (other or {}).get(n, n)) for n in names}


L2_NOTE = ("inputs larger than L2: each fragment's inputs were last touched a whole suite step "
           "(about 22 GB of traffic per GPU) earlier, L2 is 0.126 GB; no explicit flush in the "
           "timed steps")


DATA = "synthetic (seeded generators with the configs' shapes and distributions)"


def config_dict(workload, world, fragments: dict):
    """The same dict from both arms for the same workload and world size."""
    return {"workload": workload, "fragments": fragments,
            "parallelism": f"dp{world} (rows per rank fixed; dweight exchange for C1B/C4B)",
            "l2": L2_NOTE}


def reference_arm(args, rank, world):
    if rank != 0:
        return 0
    names = SUITE if args.workload == "suite" else [args.workload]
    steps, warm = max(1, args.steps), max(0, args.warmup)
    per_step = args.ref_seconds / (steps + warm + 2)
    frac = calibrate_cpu(names, per_step)
    sample = cpu_suite_sample(frac, names)
    for _ in range(warm):
        for _, _, _, fn in sample:
            fn()
    t0 = time.perf_counter()
    tot_b = 0
    for _ in range(steps):
        for _, nb, _, fn in sample:
            fn()
            tot_b += nb
    dt = time.perf_counter() - t0
    gbs = tot_b / dt / 1e9
    line = {"impl": "reference", "metric": METRIC, "value": round(gbs, 3), "unit": UNIT,
            "n_gpus": world, "steps": steps, "warmup": warm,
            "ms_per_step": round(dt / steps * 1e3, 3), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": DATA,
            "config": config_dict(args.workload, world, suite_descriptions(names)),
            "cpu_baseline": {"value": round(gbs, 3), "unit": UNIT, "cores": torch.get_num_threads(),
                             "kind": "port",
                             "sample": (f"torch-eager CPU restatement of the reference graphs "
                                        f"(oracle/fragments.py) on {frac:.4g} of each config's rows "
                                        f"per step")},
            "e2e": {"value": round(gbs, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------ parity and extra legs

def _f64_colsum(g, x, r, chunk=8192):
    """float64 column sums of g * x * r over the rows, and of the squared
    terms (for a tolerance floor on near-zero columns); torch on the GPU,
    chunked by rows."""
    N = x.shape[-1]
    g2, x2, r2 = g.reshape(-1, N), x.reshape(-1, N), r.reshape(-1)
    s = torch.zeros(N, dtype=torch.float64, device=x.device)
    q = torch.zeros_like(s)
    for i in range(0, g2.shape[0], chunk):
        t = g2[i:i + chunk].double() * x2[i:i + chunk].double() * r2[i:i + chunk, None].double()
        s += t.sum(0)
        q += t.pow(2).sum(0)
    return s, q


def _host_memory_fits(step_bytes, world, dev, avail=None):
    """Whether every rank on this host can pin its e2e buffers (about a
    step's algorithmic bytes of pinned inputs and outputs per rank) within
    75 % of the host's available memory (`avail` bytes, read from
    /proc/meminfo when not given); all ranks take the same answer."""
    local = int(os.environ.get("LOCAL_WORLD_SIZE", world))
    if avail is None:
        avail = 0
        try:
            with open("/proc/meminfo") as fh:
                for ln in fh:
                    if ln.startswith("MemAvailable:"):
                        avail = int(ln.split()[1]) * 1024
        except OSError:
            pass
    need = step_bytes * local
    ok = avail == 0 or need < 0.75 * avail  # unknown: assume it fits
    ok = _all_ok(ok, dev, world)
    why = (f"{local} ranks x {step_bytes / 1e9:.1f} GB of pinned host buffers would exceed 75% of the "
           f"{avail / 1e9:.0f} GB available on this host")
    return ok, ("" if ok else why)


def _all_ok(flag: bool, dev, world) -> bool:
    t = torch.tensor([1 if flag else 0], dtype=torch.int32, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MIN)
    return bool(t.item())


def dweight_parity(g, x, r, local, glob, world, dev):
    """The dweight a rank ends with, checked two ways:
    * against the float64 column sum over every rank's rows (rtol 1e-4, with
      a floor of 1e-4 x the column's L2 norm for near-zero columns);
    * bit for bit against the fixed rank-order sum of every rank's own
      dweight, gathered separately and reduced on this rank, and equal on
      every rank."""
    from kernelproblems_b200 import ops
    s64, q64 = _f64_colsum(g, x, r)
    if world > 1:
        dist.all_reduce(s64)
        dist.all_reduce(q64)
    got = (glob if glob is not None else local).double()
    err = (got - s64).abs()
    bound = 1e-4 * s64.abs() + 1e-4 * q64.sqrt()
    ok64 = bool((err <= bound).all().item())
    rel = float((err / s64.abs().clamp_min(1e-30)).median().item())
    out = {"vs_float64_rtol_1e-4": _all_ok(ok64, dev, world), "median_rel_err": rel}
    if world > 1:
        parts = torch.empty(world, local.numel(), dtype=torch.float32, device=dev)
        dist.all_gather_into_tensor(parts.view(-1), local.contiguous())
        ref = ops.dw_reduce(parts)
        same = torch.equal(ref, glob)
        globs = torch.empty(world, glob.numel(), dtype=torch.float32, device=dev)
        dist.all_gather_into_tensor(globs.view(-1), glob.contiguous())
        agree = all(torch.equal(globs[0], globs[i]) for i in range(world))
        out["bitwise_rank_order_sum"] = _all_ok(same, dev, world)
        out["ranks_agree_bitwise"] = _all_ok(agree, dev, world)
    return out


class L2Flush:
    """Writes a 256 MB buffer (twice the 126 MB L2) between timed reps."""

    def __init__(self, dev):
        self.buf = torch.empty(256 << 20, dtype=torch.uint8, device=dev)

    def __call__(self):
        self.buf.zero_()


def _time_reps(fn_kernels, fn_after, reps, flush, world):
    """Per rep: flush L2, then events around fn_kernels() and fn_after()
    (None: nothing).  Returns (mean kernel ms, mean total ms), max over ranks.

    One untimed rep first (a new graph's first replay uploads it), then the
    ranks line up on the host, so the first timed exchange does not absorb
    how long each rank took to get here (capturing a graph, for one, takes
    each rank a different time)."""
    flush()
    fn_kernels()
    if fn_after is not None:
        fn_after()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
        torch.cuda.synchronize()
    ka, kb, kc = [], [], []
    for _ in range(reps):
        flush()
        a, b, c = (torch.cuda.Event(enable_timing=True) for _ in range(3))
        a.record()
        fn_kernels()
        b.record()
        if fn_after is not None:
            fn_after()
        c.record()
        ka.append(a)
        kb.append(b)
        kc.append(c)
    torch.cuda.synchronize()
    k = statistics.fmean(a.elapsed_time(b) for a, b in zip(ka, kb))
    t = statistics.fmean(a.elapsed_time(c) for a, c in zip(ka, kc)) if fn_after is not None else k
    v = torch.tensor([k, t], dtype=torch.float64, device=torch.cuda.current_device())
    if world > 1:
        dist.all_reduce(v, op=dist.ReduceOp.MAX)
    return v[0].item(), v[1].item()


def _graph_of(fn):
    """fn captured into a CUDA graph after one eager warm-up call."""
    fn()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, capture_error_mode="thread_local"):
        fn()
    torch.cuda.synchronize()
    return g


def strong_scaling_leg(dev, world, rank, pg, reps=20):
    """The row-sharded configurations (C0, C1, C4 fwd and bwd) with a fixed
    total: rank r takes rows [r*M/W, (r+1)*M/W) of one global problem (the
    same seeded tensors on every rank), C1B and C4B add the dweight exchange
    (all-gather of the per-rank vectors, fixed rank-order sum).  Each rank
    also times the whole configuration alone, the 1-GPU reference of the
    efficiency.  Kernel and exchange times are reported separately; all
    times are means over reps with an L2 flush before each, max over ranks."""
    from kernelproblems_b200 import configs as cf
    from kernelproblems_b200 import ops, sharding
    flush = L2Flush(dev)
    out = {}
    for name, c in (("C0F", cf.C0), ("C1B", cf.C1), ("C4F", cf.C4), ("C4B", cf.C4)):
        M, N = c.M, c.N
        sh = cf.shard_rows(M, world, rank)
        w = cf.rmsnorm_weight(N, device=dev, seed=90)
        full = {k: cf.randn((M, N), device=dev, seed=91 + i)
                for i, k in enumerate(("x", "g", "dh") if name in ("C1B", "C4B") else ("x", "res"))}
        if name == "C4B":  # the backward's input is the forward's h and its rstd
            full["x"], _, _ = ops.add_rmsnorm_fwd(full["dh"], full["x"], w, c.eps, save_rstd=False)
        if name in ("C1B", "C4B"):
            _, full["r"] = ops.rmsnorm_fwd(full["x"], w, c.eps)

        def call(t, ws=None):
            if name == "C0F":
                return ops.rmsnorm_fwd(t["x"], w, c.eps)
            if name == "C4F":
                return ops.add_rmsnorm_fwd(t["res"], t["x"], w, c.eps)
            return ops.rmsnorm_bwd(t["g"], t["x"], t["r"], w, eps=c.eps,
                                   dres=t["dh"] if name == "C4B" else None, workspace=ws)
        rec = {"rows_total": M, "rows_per_rank_max": cf.shard_rows(M, world, 0).n}
        # the whole configuration on this GPU alone
        ws_full = torch.empty(ops.rmsnorm_bwd_workspace_bytes(M, N), dtype=torch.uint8, device=dev) \
            if name in ("C1B", "C4B") else None
        g_full = _graph_of(lambda: call(full, ws_full))
        rec["full_1gpu_ms"], _ = _time_reps(g_full.replay, None, reps, flush, world)
        del g_full, ws_full
        shard = {k: v[sh.lo:sh.hi].contiguous() for k, v in full.items()}
        del full
        torch.cuda.empty_cache()
        ws = torch.empty(max(16, ops.rmsnorm_bwd_workspace_bytes(sh.n, N)), dtype=torch.uint8, device=dev) \
            if name in ("C1B", "C4B") else None
        holder = {}

        def local():
            holder["out"] = call(shard, ws)
        g_sh = _graph_of(local)
        exchange = peer = None
        if name in ("C1B", "C4B") and world > 1:
            pbuf = torch.empty(world, N, dtype=torch.float32, device=dev)
            dwg = torch.empty(N, dtype=torch.float32, device=dev)
            dwp = torch.empty(N, dtype=torch.float32, device=dev)

            def exchange():
                dist.all_gather_into_tensor(pbuf.view(-1), holder["out"][1], group=pg)
                ops.dw_reduce(pbuf, out=dwg)
            err = ""
            try:  # the same exchange over NVLink peer memory, one launch
                peer = sharding.PeerDweightExchange(N, group=pg, device=dev)
            except Exception as e:  # every rank agrees below before using it
                err = repr(e)[:200]
            if not _all_ok(peer is not None, dev, world):
                if peer is not None:
                    peer.close()
                peer = None
                rec["exchange_peer_error"] = err or "another rank could not set up its peer buffers"
        k_ms, t_ms = _time_reps(g_sh.replay, exchange, reps, flush, world)
        if peer is not None:
            # the peer exchange has no per-call host arguments: kernel and
            # exchange are one captured graph, timed as device work
            pout = {}

            def local_and_peer():
                pout["out"] = call(shard, ws)
                peer(pout["out"][1], out=dwp)
            g_pe = _graph_of(local_and_peer)
            tp_ms, _ = _time_reps(g_pe.replay, None, reps, flush, world)
            torch.cuda.synchronize()
            rec["exchange_peer_ms"] = round(tp_ms - k_ms, 4)
            rec["ms_peer"] = round(tp_ms, 4)
            rec["efficiency_peer"] = round(rec["full_1gpu_ms"] / (world * tp_ms), 3)
            same = torch.equal(dwp, dwg) and torch.equal(pout["out"][1], holder["out"][1])
            rec["peer_equals_nccl_path_bitwise"] = _all_ok(same, dev, world)
            del g_pe
            peer.close()
        nbytes = {"C0F": cf.bytes_rmsnorm_fwd, "C1B": cf.bytes_rmsnorm_bwd,
                  "C4F": cf.bytes_add_rmsnorm_fwd, "C4B": cf.bytes_add_rmsnorm_bwd}[name](M, N)
        rec.update({"kernel_ms": round(k_ms, 4), "exchange_ms": round(t_ms - k_ms, 4),
                    "ms": round(t_ms, 4), "full_1gpu_ms": round(rec["full_1gpu_ms"], 4),
                    "tokens_per_s": round(M / (t_ms * 1e-3)),
                    "GB/s_aggregate": round(nbytes / (t_ms * 1e-3) / 1e9, 1),
                    "speedup_vs_1gpu": round(rec["full_1gpu_ms"] / t_ms, 3),
                    "efficiency": round(rec["full_1gpu_ms"] / (world * t_ms), 3)})
        if name in ("C1B", "C4B"):
            torch.cuda.synchronize()
            rec["parity"] = dweight_parity(shard["g"], shard["x"], shard["r"], holder["out"][1],
                                           dwg if world > 1 else None, world, dev)
        out[name] = rec
        del g_sh, shard, ws, holder
        torch.cuda.empty_cache()
    tot_full = sum(v["full_1gpu_ms"] for v in out.values())
    tot = sum(v["ms"] for v in out.values())
    tot_peer = sum(v.get("ms_peer", v["ms"]) for v in out.values())
    return {"fragments": out, "sum_ms": round(tot, 4), "sum_full_1gpu_ms": round(tot_full, 4),
            "efficiency": round(tot_full / (world * tot), 3),
            "efficiency_peer_exchange": round(tot_full / (world * tot_peer), 3),
            "method": ("one global problem per configuration (same seeds on every rank), rank r "
                       "takes its contiguous rows; kernels replayed from a CUDA graph, exchange "
                       "(NCCL all-gather + fixed-order sum) launched eagerly after the replay; *_peer: "
                       "the NVLink peer-memory exchange captured with the kernel in one graph; "
                       "one untimed rep, ranks lined up on the host, then L2 flushed before each of "
                       f"{reps} reps; efficiency = full-config 1-GPU ms / (N x sharded ms)")}


def emb_vp_leg(dev, world, rank, pg, steps=30):
    """Vocab-parallel embedding at the C2 shapes: rank r holds table rows
    [lo_r, hi_r) (the 8-way split of the reference's FSDP layout at N = 8);
    forward = masked gather of the replicated ids + NCCL all-reduce of the
    bf16 [32768, 4096] output, backward = this rank's fp32 table-gradient
    shard.  Gather, all-reduce and backward are timed separately (events per
    step; max over ranks).  Parity: the all-reduced output equals a full
    gather from the whole table bit for bit (rank 0 rebuilds the whole table
    from every shard's seed), and each rank's gradient shard equals the same
    rows of the unsharded backward."""
    from kernelproblems_b200 import configs as cf
    from kernelproblems_b200 import ops, sharding
    c = cf.C2
    sh = cf.shard_rows(c.vocab, world, rank)
    ids = cf.embedding_ids(c, device=dev)
    table = cf.randn((sh.n, c.dim), std=0.02, device=dev, seed=7 + 1000 * sh.lo)
    g = cf.randn((*c.batch, c.dim), device=dev, seed=8)
    Gs = torch.empty(sh.n, c.dim, dtype=torch.float32, device=dev)
    ws = torch.empty(max(16, ops._lib.load().frag_embedding_bwd_workspace_bytes(c.T, sh.n)),
                     dtype=torch.uint8, device=dev)
    out = torch.empty(*c.batch, c.dim, dtype=torch.bfloat16, device=dev)

    def bwd():
        sharding.embedding_bwd_vocab_parallel(
            g, ids, sh.lo, sh.n, c.vocab,
            bwd_fn=lambda *a, **k: ops.embedding_bwd(*a, **k, out=Gs, workspace=ws))
    for _ in range(3):
        ops.embedding_fwd(ids, table, vocab_lo=sh.lo, vocab_total=c.vocab, out=out)
        if world > 1:
            dist.all_reduce(out, group=pg)
        bwd()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    evs = []
    for _ in range(steps):
        e = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
        e[0].record()
        ops.embedding_fwd(ids, table, vocab_lo=sh.lo, vocab_total=c.vocab, out=out)
        e[1].record()
        if world > 1:
            dist.all_reduce(out, group=pg)
        e[2].record()
        bwd()
        e[3].record()
        evs.append(e)
    torch.cuda.synchronize()
    gather = statistics.fmean(e[0].elapsed_time(e[1]) for e in evs)
    ar = statistics.fmean(e[1].elapsed_time(e[2]) for e in evs)
    bw = statistics.fmean(e[2].elapsed_time(e[3]) for e in evs)
    total = evs[0][0].elapsed_time(evs[-1][3]) / steps
    v = torch.tensor([gather, ar, bw, total], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(v, op=dist.ReduceOp.MAX)
    gather, ar, bw, total = v.tolist()
    # parity (outside the timed region)
    parts = [cf.randn((cf.shard_rows(c.vocab, world, r).n, c.dim), std=0.02, device=dev,
                      seed=7 + 1000 * cf.shard_rows(c.vocab, world, r).lo) for r in range(world)] \
        if rank == 0 else None
    fwd_ok = True
    if rank == 0:
        full = torch.cat(parts)
        del parts
        fwd_ok = torch.equal(out, ops.embedding_fwd(ids, full))
        del full
    Gfull = ops.embedding_bwd(g, ids, c.vocab)
    bwd_ok = torch.equal(Gs, Gfull[sh.lo:sh.hi])
    del Gfull
    torch.cuda.empty_cache()
    out_bytes = c.T * c.dim * cf.BF16
    peer = _emb_vp_peer(dev, world, pg, ids, table, sh, c, out, gather + ar, steps)
    nb = cf.bytes_embedding_fwd(c.T, c.dim) + cf.bytes_embedding_bwd(c.T, c.dim, c.vocab)
    return {"ms_per_step": round(total, 4), "gather_ms": round(gather, 4),
            "allreduce_ms": round(ar, 4), "bwd_shard_ms": round(bw, 4),
            "allreduce_bytes": out_bytes,
            "allreduce_busbw_GBs": (round(2 * (world - 1) / world * out_bytes / (ar * 1e-3) / 1e9, 1)
                                    if world > 1 else None),
            "GB/s_aggregate": round(nb / (total * 1e-3) / 1e9, 1),
            "tokens_per_s": round(c.T / (total * 1e-3)), "steps": steps,
            "parity": {"fwd_bit_exact_vs_full_gather": _all_ok(fwd_ok, dev, world),
                       "bwd_shard_equals_unsharded_rows": _all_ok(bwd_ok, dev, world)},
            "fused_peer_fwd": peer,
            "layout": f"vocab{world}: rank r owns table rows [r*V/W, (r+1)*V/W), ids and grad replicated",
            "scaling": "strong (fixed 32768 tokens, table split over ranks)"}


def _emb_vp_peer(dev, world, pg, ids, table, sh, c, ref_out, nccl_fwd_ms, steps):
    """The same vocab-parallel forward with the exchange fused into the gather
    over NVLink peer memory (sharding.PeerVocabParallelEmbedding): forward ms
    (events, mean, max over ranks) and bit-exact parity with the NCCL path's
    output (itself checked against the full gather)."""
    from kernelproblems_b200 import sharding
    pe, err = None, ""
    try:
        pe = sharding.PeerVocabParallelEmbedding(c.T, c.dim, group=pg, device=dev)
    except Exception as e:  # reported; every rank agrees below before using it
        err = repr(e)[:200]
    if not _all_ok(pe is not None, dev, world):
        if pe is not None:
            pe.close()
        return {"error": err or "another rank could not set up its peer buffers"}
    try:
        for _ in range(3):
            pe(ids, table, sh.lo, c.vocab)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        evs = []
        for _ in range(steps):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            o = pe(ids, table, sh.lo, c.vocab)
            b.record()
            evs.append((a, b))
        torch.cuda.synchronize()
        ms = torch.tensor([statistics.fmean(a.elapsed_time(b) for a, b in evs)], dtype=torch.float64,
                          device=dev)
        if world > 1:
            dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        ms = ms.item()
        same = torch.equal(o.view_as(ref_out), ref_out)
        from kernelproblems_b200 import _lib as L
        flags = L.load().frag_device_errors(1)
        out_bytes = c.T * c.dim * 2
        return {"fwd_ms": round(ms, 4),
                "nvlink_GBs_per_rank_out": (round((world - 1) / world * out_bytes / (ms * 1e-3) / 1e9, 1)
                                            if world > 1 else None),
                "speedup_vs_gather_plus_allreduce": round(nccl_fwd_ms / ms, 3),
                "parity_bit_exact_vs_nccl_path": _all_ok(same and flags == 0, dev, world),
                "steps": steps,
                "design": ("owner gathers each row once and stores it into every rank's output over "
                           "CUDA IPC peer mappings with plain stores; bounded flag barriers (entry, exit)")}
    finally:
        pe.close()


def _freqs_cis(dim, end, theta, dev):
    """torchtitan's precompute_freqs_cis: complex64 [end, dim/2]."""
    f = 1.0 / (theta ** (torch.arange(0, dim, 2, device=dev)[: dim // 2].float() / dim))
    t = torch.arange(end, device=dev, dtype=torch.float32)
    return torch.polar(torch.ones(end, dim // 2, device=dev), torch.outer(t, f))


def problem_inputs(cfg, dev):
    """Inputs of the reference problem(s) a configuration comes from, in the
    problems' own formats (get_inputs() order) at the configuration's size,
    seeded: {problem: [inputs]}, and the algorithmic bytes of one call under
    the problems' own contracts."""
    from kernelproblems_b200 import configs as cf
    if cfg == "C0F":
        c = cf.C0
        return {"v8/f4e9e58fef73": [cf.randn(c.shape, device=dev, seed=1),
                                    cf.rmsnorm_weight(c.N, device=dev, seed=2)]}, \
            cf.bytes_rmsnorm_fwd(c.M, c.N)
    if cfg == "C1B":
        c = cf.C1
        return {"v7/45990c83cfd6": [cf.randn(c.shape, device=dev, seed=3),
                                    cf.rmsnorm_weight(c.N, device=dev, seed=4),
                                    cf.randn(c.shape, device=dev, seed=5)]}, \
            3 * c.M * c.N * 2 + 4 * c.N  # x, dy, dx; w, dw (bf16): rstd recomputed
    if cfg in ("C2F", "C2B"):
        c = cf.C2
        ids = cf.embedding_ids(c, device=dev)
        if cfg == "C2F":
            return {"v7/1e49beb8a123": [cf.randn((c.vocab * c.dim,), std=0.02, device=dev, seed=6),
                                        ids]}, cf.bytes_embedding_fwd(c.T, c.dim)
        return {"v7/a12a160cb11b": [cf.randn((*c.batch, c.dim), device=dev, seed=7), ids]}, \
            cf.bytes_embedding_bwd(c.T, c.dim, c.vocab)
    if cfg in ("C3F", "C3B"):
        c = cf.C3
        T = c.T
        pos = cf.rope_positions(c, device=dev).view(1, T)
        if cfg == "C3F":
            fr = _freqs_cis(c.D, c.S, c.theta, dev)
            return {"v8/c8c60d8f7015": [pos.to(torch.int32), fr,
                                        cf.randn((T, c.Hq * c.D), device=dev, seed=8),
                                        cf.randn((T, c.Hk * c.D), device=dev, seed=9)]}, \
                cf.bytes_rope(T, c.Hq, c.Hk, c.D) - T * 8 + T * 4 + fr.numel() * 8
        conj = _freqs_cis(c.D, c.S, c.theta, dev)[pos.view(-1)].conj().resolve_conj() \
            .view(1, T, 1, c.D // 2).contiguous()
        gq = cf.randn((T * c.Hq * c.D,), device=dev, seed=10).as_strided(
            [1, c.Hq, T, c.D], [T * c.Hq * c.D, c.D, c.Hq * c.D, 1])
        gk = cf.randn((T * c.Hk * c.D,), device=dev, seed=11).as_strided(
            [1, c.Hk, T, c.D], [T * c.Hk * c.D, c.D, c.Hk * c.D, 1])
        return {"v7/bfe872e373e4": [gq, conj], "v7/5c65f62b0422": [gk, conj]}, \
            4 * T * (c.Hq + c.Hk) * c.D + 2 * T * (c.D // 2) * 8
    c = cf.C4
    M, N = c.M, c.N
    w = cf.rmsnorm_weight(N, device=dev, seed=12)
    if cfg == "C4F":
        return {"v8/7884328a5557": [cf.randn((M, N), device=dev, seed=13),
                                    cf.randn((1, M, N), device=dev, seed=14), w]}, \
            3 * M * N * 2 + 2 * N  # res, x read; y written (the problem returns y only)
    h = cf.randn((1, M, N), device=dev, seed=15)
    r = torch.rsqrt(h.float().pow(2).mean(-1, keepdim=True) + c.eps)
    return {"v7/7f544ceb2120": [cf.randn((M, N), device=dev, seed=16),
                                cf.randn((1, M, N), device=dev, seed=17), h, r, w,
                                cf.randn((1, M, N), device=dev, seed=18)]}, \
        5 * M * N * 2 + 4 * M + 2 * N + 4 * N


def pcie_leg(dev, world, nbytes=1 << 30, reps=5):
    """Host <-> device copy bandwidth of this rank alone and with every rank
    copying at once: 1 GiB pinned buffers, H2D, D2H, and both directions at
    the same time on two streams (GB/s per rank, min over ranks)."""
    h = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
    h2 = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
    d = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    d2 = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    s1, s2 = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    out = {}
    for name in ("h2d", "d2h", "both"):
        d.copy_(h, non_blocking=True)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        t0 = time.perf_counter()
        for _ in range(reps):
            if name in ("h2d", "both"):
                with torch.cuda.stream(s1):
                    d.copy_(h, non_blocking=True)
            if name in ("d2h", "both"):
                with torch.cuda.stream(s2):
                    h2.copy_(d2, non_blocking=True)
        torch.cuda.synchronize()
        dt = time.perf_counter() - t0
        gbs = torch.tensor([nbytes * reps * (2 if name == "both" else 1) / dt / 1e9], device=dev)
        if world > 1:
            dist.all_reduce(gbs, op=dist.ReduceOp.MIN)
        out[name + "_GBs_per_rank"] = round(gbs.item(), 1)
    out["note"] = ("1 GiB pinned copies, every rank at once (wall clock over 5 copies, min over ranks); "
                   "PCIe Gen5 x16 is 64 GB/s per direction nominal")
    return out


def e2e_dropin(dev, world, reps=3):
    """Each configuration's reference problem(s) through this library's
    drop-in kernel_function (kernelproblems_b200.problems, the reference's own
    calling contract): inputs uploaded from pinned host memory, the call,
    every output copied back to pinned host memory, all inside the events
    (mean of `reps` after a warm-up).  Configurations run one at a time; a
    step is their sum."""
    from kernelproblems_b200 import problems
    per, tot_ms, tot_b, tot_in, tot_out = {}, 0.0, 0, 0, 0
    for cfg in SUITE:
        probs, nbytes = problem_inputs(cfg, dev)
        host = {p: [t.cpu().pin_memory() for t in inp] for p, inp in probs.items()}
        del probs
        torch.cuda.empty_cache()
        outs_h = {}

        def one():
            nin = nout = 0
            for p, hin in host.items():
                xs = [t.to(dev, non_blocking=True) for t in hin]
                o = problems.get_kernel_function(p)(*xs)
                o = o if isinstance(o, (tuple, list)) else (o,)
                bufs = outs_h.setdefault(p, [torch.empty(t.shape, dtype=t.dtype, pin_memory=True) for t in o])
                for b, t in zip(bufs, o):
                    b.copy_(t, non_blocking=True)
                nin += sum(t.numel() * t.element_size() for t in hin)
                nout += sum(t.numel() * t.element_size() for t in o)
            return nin, nout
        one()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(reps):
            nin, nout = one()
        b.record()
        torch.cuda.synchronize()
        ms = torch.tensor([a.elapsed_time(b) / reps], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        ms = ms.item()
        per[cfg] = {"problems": list(host), "ms": round(ms, 3), "h2d_bytes": nin, "d2h_bytes": nout,
                    "GB/s_algorithmic": round(nbytes / (ms * 1e-3) / 1e9, 1)}
        tot_ms += ms
        tot_b += nbytes
        tot_in += nin
        tot_out += nout
        del host, outs_h
        torch.cuda.empty_cache()
    return {"value": round(world * tot_b / (tot_ms * 1e-3) / 1e9, 2), "unit": UNIT,
            "ms_per_step": round(tot_ms, 3), "h2d_bytes_per_step": tot_in, "d2h_bytes_per_step": tot_out,
            "fragments": per,
            "path": ("kernelproblems_b200.problems.get_kernel_function(problem)(*inputs) with inputs "
                     "from pinned host memory and outputs copied back, the problems' own contracts "
                     "and algorithmic bytes (as in triton_reference)")}


def triton_leg(dev, reps=10):
    """The reference's Triton drop-ins (oracle/_ref/triton, fetched by
    oracle/triton_ref.py) and this library's drop-ins for the same problems,
    on the same inputs at each configuration's size, each call replayed from
    a CUDA graph with an L2 flush before each rep (mean ms).  Parity: each
    output of the reference kernel against ours (bf16 outputs atol 1e-2 /
    rtol 1.6e-2, the embedding gather bit for bit, fp32 table gradient and
    dweight rtol 1e-4 with a small floor)."""
    from oracle import triton_ref
    if not triton_ref.available():
        return {"unavailable": "oracle/_ref/triton is missing (python oracle/triton_ref.py --reference <checkout>)"}
    from kernelproblems_b200 import configs as cf
    from kernelproblems_b200 import problems
    flush = L2Flush(dev)
    res = {}

    def close(a, b, cfg, addend=None):
        """a (reference kernel) against b (ours)."""
        if cfg == "C2F":
            return bool(torch.equal(a, b))
        if a.dtype != b.dtype or a.shape != b.shape:
            return False
        af, bf = a.double(), b.double()
        if a.dtype == torch.float32:  # rstd, fp32 dweight, fp32 table gradient
            atol = 1e-5 if cfg == "C2B" else 1e-4 * bf.abs().mean().item()
            return bool(((af - bf).abs() <= 1e-4 * bf.abs() + atol).all())
        tol = 1e-2 + 1.6e-2 * bf.abs()
        if addend is not None:
            # bf16(dres + dx): the reference kernel adds the unrounded dx, the
            # graph (and this library) bf16(dx); one ulp of |dx| may survive
            # cancellation
            t = (bf - addend.double()).abs().clamp_min(2.0 ** -126)
            tol = tol + torch.exp2(torch.floor(torch.log2(t)) - 7)
        return bool(((af - bf).abs() <= tol).all())

    for cfg in ("C0F", "C1B", "C2F", "C2B", "C3F", "C3B", "C4F", "C4B"):
        probs, nbytes = problem_inputs(cfg, dev)
        rec = {"problems": list(probs), "bytes": nbytes}
        ours_ms = ref_ms = 0.0
        parity = True
        for prob, inp in probs.items():
            f_ours = problems.get_kernel_function(prob)
            f_ref = triton_ref.kernel_function(prob)
            o1 = f_ours(*inp)
            o2 = f_ref(*inp)
            torch.cuda.synchronize()
            o1 = o1 if isinstance(o1, (tuple, list)) else (o1,)
            o2 = o2 if isinstance(o2, (tuple, list)) else (o2,)
            addend = inp[5] if cfg == "C4B" else None
            parity = parity and len(o1) == len(o2) and all(
                close(b, a, cfg, addend if a.dtype == torch.bfloat16 else None)
                for a, b in zip(o1, o2))
            del o1, o2
            g1 = _graph_of(lambda: f_ours(*inp))
            g2 = _graph_of(lambda: f_ref(*inp))
            ours_ms += _time_reps(g1.replay, None, reps, flush, 1)[0]
            ref_ms += _time_reps(g2.replay, None, reps, flush, 1)[0]
            del g1, g2
        rec.update({"ours_ms": round(ours_ms, 4), "triton_ms": round(ref_ms, 4),
                    "ours_GB/s": round(nbytes / (ours_ms * 1e-3) / 1e9, 1),
                    "triton_GB/s": round(nbytes / (ref_ms * 1e-3) / 1e9, 1),
                    "speedup_vs_triton": round(ref_ms / ours_ms, 3),
                    "parity_triton_vs_ours": parity})
        res[cfg] = rec
        del probs
        torch.cuda.empty_cache()
    return {"fragments": res,
            "method": ("each problem's reference kernel_function (oracle/_ref/triton, size patches "
                       "listed in oracle/triton_ref.py) and this library's drop-in for the same "
                       "problem on the same inputs at the configuration's size; one call per CUDA "
                       f"graph, L2 flushed before each of {reps} reps; the problems' own contracts "
                       "(C1B recomputes rstd and returns a bf16 dweight, C3 is the interleaved "
                       "complex layout with a freqs table, C4F returns y only, C4B sums two "
                       "gradients)")}


def ours_arm(args, rank, local_rank, world):
    from kernelproblems_b200 import _lib
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    pg = None
    if world > 1:
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
        pg = dist.group.WORLD
    _lib.load()
    if args.workload == "emb_vp":
        line = {"metric": METRIC, "unit": UNIT, "n_gpus": world, "emb_vp": emb_vp_leg(dev, world, rank, pg,
                                                                                     args.steps)}
        line["value"] = line["emb_vp"]["GB/s_aggregate"]
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        if rank == 0:
            print(json.dumps(line), flush=True)
        return 0
    names = {"suite": SUITE, "next": NEXT}.get(args.workload, [args.workload])
    frags = build_suite(dev, world, rank, names, pg, args.rows_frac, exchange=args.exchange)
    step = Step(frags, not args.no_graphs)
    step_bytes = sum(f.bytes for f in frags)
    stream = torch.cuda.current_stream(dev)

    if world > 1:
        dist.barrier()  # the first exchange's bounded waits start with every rank here
    for _ in range(max(3, args.warmup)):
        step.run()
    step.join()
    torch.cuda.synchronize()
    K = args.steps
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    clocks = ClockSampler(dev, enabled=(rank == 0 and not args.no_clocks))
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clocks.start()
    t_start.record(stream)
    for _ in range(K):
        step.run()
    step.join()  # the last step's exchange is inside the timed region
    t_end.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    if world > 1:
        dist.barrier()
    total_ms = t_start.elapsed_time(t_end)
    # dweight parity of the timed step's results (every rank, same order)
    parity = {}
    for f in frags:
        chk = getattr(f, "dw_check", None)
        if chk is not None:
            parity[f.name] = dweight_parity(chk["g"], chk["x"], chk["r"], chk["local"](),
                                            chk["glob"]() if chk["glob"] else None, world, dev)
    # per-fragment / per-stage breakdown: the same step replayed R more times,
    # read from the events inside the step after each replay (exchanges inline)
    R = max(5, min(K, 30))
    frag_ms = {f.name: [] for f in frags}
    ex_ms = {f.name: [] for f in frags}
    stage_ms = {f.name: [[] for _ in f.stages] for f in frags}
    for _ in range(R):
        if world > 1:
            dist.barrier()  # start every breakdown replay together, so no rank's
            torch.cuda.synchronize()  # exchange absorbs another rank's skew
        step.run_instrumented()
        torch.cuda.synchronize()
        for f in frags:
            st = [f.ev[i].elapsed_time(f.ev[i + 1]) for i in range(len(f.stages))]
            frag_ms[f.name].append(f.ev[0].elapsed_time(f.ev[-1]))
            if f.ev_end is not None:
                ex_ms[f.name].append(f.ev[-1].elapsed_time(f.ev_end))
            for i, v in enumerate(st):
                stage_ms[f.name][i].append(v)
    # max over ranks
    tmax = torch.tensor([total_ms] + [statistics.fmean(frag_ms[f.name]) for f in frags]
                        + [statistics.fmean(ex_ms[f.name]) if ex_ms[f.name] else 0.0 for f in frags],
                        dtype=torch.float64, device=dev)
    tmin = tmax.clone()
    if world > 1:
        dist.all_reduce(tmax, op=dist.ReduceOp.MAX)
        dist.all_reduce(tmin, op=dist.ReduceOp.MIN)
    tmin = tmin.tolist()
    tmax = tmax.tolist()
    ms_step = tmax[0] / K
    value = world * step_bytes / (ms_step * 1e-3) / 1e9
    tokens = sum(f.tokens for f in frags)
    peak, peak_note = measured_peak()
    nf = len(frags)

    fr = {}
    for i, f in enumerate(frags):
        ms = tmax[1 + i]
        fr[f.name] = {"ms": round(ms, 4), "GB/s_per_gpu": round(f.bytes / (ms * 1e-3) / 1e9, 1),
                      "pct_of_8TBs": round(100 * f.bytes / (ms * 1e-3) / 1e9 / NOMINAL_HBM_GBS, 1),
                      "frac_of_measured": round(f.bytes / (ms * 1e-3) / 1e9 / peak, 3),
                      "tokens_per_s": round(world * f.tokens / (ms * 1e-3)),
                      "bytes": f.bytes, "tokens": f.tokens,
                      "stages_ms": {lab: round(statistics.fmean(stage_ms[f.name][si]), 4)
                                    for si, (lab, _) in enumerate(f.stages)}}
        if f.exchange is not None:
            fr[f.name]["exchange_ms_inline"] = round(tmax[1 + nf + i], 4)
    dom = next((f for f in frags if f.name == DOMINANT), frags[0])
    main_ms = statistics.fmean(stage_ms[dom.name][0])
    achieved = dom.bytes / (main_ms * 1e-3) / 1e9
    traffic = None
    tinfo = profile_traffic()
    if tinfo and tinfo.get("fragment") == dom.name:
        traffic = tinfo.get("dram_bytes_per_launch")
    roof = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
            "frac": round(achieved / peak, 4), "traffic": traffic,
            "kernel": f"{dom.name} {dom.stages[0][0]} (main kernel of the fragment)",
            "algorithmic_bytes_per_launch": dom.bytes, "launch_ms": round(main_ms, 4),
            "peak_source": peak_note, "pct_of_8TBs": round(100 * achieved / NOMINAL_HBM_GBS, 1)}

    # graph kernel nodes (ours and the sort's) + the eager dw_reduce of each exchange
    n_ex = sum(1 for f in frags if f.exchange is not None)
    launches = (step.kernel_nodes + n_ex) * K if step.kernel_nodes is not None else None
    line = {"metric": METRIC, "value": round(value, 1), "unit": UNIT, "n_gpus": world,
            "steps": K, "warmup": max(3, args.warmup), "ms_per_step": round(ms_step, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": DATA,
            "config": config_dict(args.workload, world,
                                  suite_descriptions([f.name for f in frags],
                                                     {f.name: f.desc for f in frags})),
            "timed_region_ms": round(total_ms, 2),
            "pct_of_8TBs_per_gpu": round(100 * value / world / NOMINAL_HBM_GBS, 1),
            "frac_of_measured_per_gpu": round(value / world / peak, 3),
            "tokens_per_s_sum_over_fragments": round(world * tokens / (ms_step * 1e-3)),
            "fragments": fr, "roofline": roof, "clocks": clk, "gpu_launches": launches,
            "parity": parity}
    if world > 1:
        line["dweight_exchange"] = {f.name: f.exchange_kind for f in frags if getattr(f, "exchange_kind", None)}
        # the spread of the per-rank figures behind the maxima above
        line["rank_spread"] = {"ms_per_step_min": round(tmin[0] / K, 4), "ms_per_step_max": round(ms_step, 4),
                               "fragment_ms_min": {f.name: round(tmin[1 + i], 4) for i, f in enumerate(frags)}}
    step.release()
    if args.workload == "suite" and args.rows_frac == 1.0 and not args.no_extra:
        # the row-sharded configurations at a fixed total (strong scaling), the
        # vocab-parallel embedding, and (one GPU) the reference's Triton kernels
        line["strong_scaling"] = strong_scaling_leg(dev, world, rank, pg)
        line["emb_vp"] = emb_vp_leg(dev, world, rank, pg)
        if world == 1:
            line["triton_reference"] = triton_leg(dev)

    # e2e through the public API with host buffers (every step: H2D inputs, D2H outputs)
    fits, why = _host_memory_fits(step_bytes, world, dev)
    if not args.no_e2e and not fits:
        line["e2e"] = {"value": None, "unit": UNIT, "skipped": why}
    elif not args.no_e2e:
        line["e2e"] = e2e_measure(frags, args.e2e_steps, world, dev, step_bytes)
        if args.workload == "suite" and args.rows_frac == 1.0 and not args.no_extra:
            line["e2e"]["pcie"] = pcie_leg(dev, world)
            if world == 1:  # the same per-rank path at every N; at N>1 it only adds host contention
                line["e2e"]["dropin"] = e2e_dropin(dev, world)
    if rank == 0 and world == 1 and not args.no_cpu_baseline and set(names) <= set(SUITE):
        line["cpu_baseline"] = cpu_baseline(names, args.cpu_seconds)
    for f in frags:  # collective: every rank holds the same peer objects
        if getattr(f, "peer", None) is not None:
            f.peer.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)
        if args.json_out:
            Path(args.json_out).write_text(json.dumps(line, indent=1))
    return 0


def e2e_measure(frags, steps, world, dev, step_bytes):
    """Every step: each fragment's inputs uploaded from pinned host memory, the
    public API call, every output read back into pinned host memory.  Uploads
    and read-backs run on their own streams (see _e2e_call), so one
    fragment's read-back overlaps the next fragment's kernels and upload."""
    global _E2E_PIPE
    hosts = {}
    for f in frags:
        # straight into pinned memory (no pageable copy in between: at 8 ranks
        # per host the inputs alone are ~95 GB)
        hosts[f.name] = {"in": {k: torch.empty(v.shape, dtype=v.dtype, pin_memory=True).copy_(v.detach())
                                for k, v in f.host.items()}, "out": {}}
    stream = torch.cuda.current_stream(dev)
    h2d_s = torch.cuda.Stream(dev)
    d2h_s = torch.cuda.Stream(dev)
    _E2E_PIPE = (h2d_s, d2h_s)
    try:
        # warm-up (allocator, pinned output buffers)
        for f in frags:
            f.e2e(hosts[f.name])
            ex = getattr(f, "exchange_e2e", None) or f.exchange
            if ex is not None:
                ex()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        h2d = d2h = 0
        a.record(stream)
        h2d_s.wait_stream(stream)  # no copy starts before the start event
        d2h_s.wait_stream(stream)
        for _ in range(steps):
            h2d = d2h = 0
            for f in frags:
                i, o = f.e2e(hosts[f.name])
                ex = getattr(f, "exchange_e2e", None) or f.exchange
                if ex is not None:
                    ex()
                h2d += i
                d2h += o
        stream.wait_stream(h2d_s)  # the end event follows every copy
        stream.wait_stream(d2h_s)
        b.record(stream)
        torch.cuda.synchronize()
    finally:
        _E2E_PIPE = None
    ms = a.elapsed_time(b) / steps
    t = torch.tensor([ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = t.item()
    return {"value": round(world * step_bytes / (ms * 1e-3) / 1e9, 2), "unit": UNIT,
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": round(ms, 3),
            "steps": steps,
            "path": "kernelproblems_b200.ops public API, inputs from pinned host memory, "
                    "every output copied back to pinned host memory; uploads and read-backs on "
                    "their own streams, overlapping neighbouring fragments' kernels"}


def main(argv=None):
    args = parse_args(argv)
    rank, local_rank, world = env_rank()
    if args.gpus != world and world == 1 and args.gpus > 1:
        print(json.dumps({"error": f"--gpus {args.gpus} needs torchrun with {args.gpus} processes"}))
        return 2
    if args.impl == "reference":
        return reference_arm(args, rank, world)
    return ours_arm(args, rank, local_rank, world)


if __name__ == "__main__":
    sys.exit(main())
