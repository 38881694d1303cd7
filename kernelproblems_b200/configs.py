"""The five workload configurations of the fragment suite, their seeded
synthetic inputs, and the algorithmic HBM bytes each fragment call must move.

Shapes and value distributions follow the benchmark definition:
  C0 RMSNorm fwd:        x [4,2048,4096] ~N(0,1), w = 1 + 0.1 N(0,1), eps 1e-6
  C1 RMSNorm bwd:        C0 plus grad_out ~N(0,1) and the saved rstd
  C2 embedding fwd/bwd:  ids [8,4096] int64, 95% uniform over 128256 rows and
                         5% from a fixed seeded set of 100 frequent ids;
                         table [128256,4096] ~N(0,0.02); grad_out [8,4096,4096]
  C3 RoPE fwd/bwd (neox): q [8,4096,32,128], k [8,4096,8,128] ~N(0,1),
                         positions arange(4096) per batch, theta 5e5
  C4 residual add + RMSNorm fwd/bwd: res, x [16,8192,8192] ~N(0,1),
                         w = 1 + 0.1 N(0,1), eps 1e-5
The reference (SherlockNoMad/KernelProblems) ships no data: its own inputs are
unseeded torch.randn / randint (e.g. v7/1e49beb8a123/problem.py:27-29), so
these seeded generators stand in for it.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import torch

BF16 = 2
F32 = 4
I64 = 8


@dataclass(frozen=True)
class RMSNormCfg:
    name: str
    shape: tuple[int, ...]
    eps: float

    @property
    def M(self) -> int:
        m = 1
        for s in self.shape[:-1]:
            m *= s
        return m

    @property
    def N(self) -> int:
        return self.shape[-1]


@dataclass(frozen=True)
class EmbeddingCfg:
    name: str
    batch: tuple[int, int]
    vocab: int
    dim: int
    hot_ids: int = 100
    hot_frac: float = 0.05
    shards: int = 8

    @property
    def T(self) -> int:
        return self.batch[0] * self.batch[1]


@dataclass(frozen=True)
class RopeCfg:
    name: str
    B: int
    S: int
    Hq: int
    Hk: int
    D: int
    theta: float

    @property
    def T(self) -> int:
        return self.B * self.S


C0 = RMSNormCfg("C0 rmsnorm_fwd x[4,2048,4096] eps=1e-6", (4, 2048, 4096), 1e-6)
C1 = RMSNormCfg("C1 rmsnorm_bwd x,grad[4,2048,4096]", (4, 2048, 4096), 1e-6)
C2 = EmbeddingCfg("C2 embedding ids[8,4096] table[128256,4096]", (8, 4096), 128256, 4096)
C3 = RopeCfg("C3 rope_neox q[8,4096,32,128] k[8,4096,8,128] theta=5e5", 8, 4096, 32, 8, 128, 500000.0)
C4 = RMSNormCfg("C4 add_rmsnorm res,x[16,8192,8192] eps=1e-5", (16, 8192, 8192), 1e-5)

CONFIGS = {"C0": C0, "C1": C1, "C2": C2, "C3": C3, "C4": C4}


# ------------------------------------------------------------ algorithmic bytes
# Every tensor a call must read or write, counted once.

def bytes_rmsnorm_fwd(M: int, N: int, rstd: bool = True) -> int:
    return 2 * M * N * BF16 + N * BF16 + (M * F32 if rstd else 0)


def bytes_rmsnorm_bwd(M: int, N: int) -> int:
    # x, dy read; dx written; rstd, w read; dw written (fp32)
    return 3 * M * N * BF16 + M * F32 + N * BF16 + N * F32


def bytes_add_rmsnorm_fwd(M: int, N: int, rstd: bool = True) -> int:
    # res, x read; h, y written
    return 4 * M * N * BF16 + N * BF16 + (M * F32 if rstd else 0)


def bytes_add_rmsnorm_bwd(M: int, N: int) -> int:
    # dy, dh, h read; d_res written; rstd, w read; dw written (fp32)
    return 4 * M * N * BF16 + M * F32 + N * BF16 + N * F32


def bytes_embedding_fwd(T: int, D: int) -> int:
    return T * I64 + 2 * T * D * BF16


def bytes_embedding_bwd(T: int, D: int, rows: int) -> int:
    return T * D * BF16 + T * I64 + rows * D * F32


def bytes_rmsnorm_embedding_bwd(T: int, D: int, rows: int, n_dy: int = 3, dres: bool = True,
                                y: bool = True) -> int:
    # x, the dy terms and dres read; w, ids read; y (recomputed forward) and
    # the fp32 table gradient and dweight written.  d_emb is not counted: the
    # fused kernel never stores it.
    return ((1 + n_dy + (1 if dres else 0) + (1 if y else 0)) * T * D * BF16 + D * BF16 + T * I64
            + rows * D * F32 + D * F32)


def bytes_rmsnorm_fwd_bwd(M: int, N: int, n_x: int, n_dy: int, dres: bool, y: bool) -> int:
    # the forward recomputed in the backward: x terms, dy terms and dres read;
    # y (when returned) and dx written; w read; dw written (fp32)
    rows = n_x + n_dy + (1 if dres else 0) + (1 if y else 0) + 1
    return rows * M * N * BF16 + N * BF16 + N * F32


def bytes_add_rmsnorm_unshard(M: int, N: int, world: int, shard: int) -> int:
    # res, x read; y written (h and rstd are not outputs); the weight gathered
    # from `world` strided pieces (read + write); the table copied out of the
    # all-gather buffer (read + write of world * shard elements)
    return 3 * M * N * BF16 + 2 * N * BF16 + 2 * world * shard * BF16


def bytes_rope(T: int, Hq: int, Hk: int, D: int) -> int:
    return 2 * T * (Hq + Hk) * D * BF16 + T * I64


# ------------------------------------------------------------- input generation

def _gen(device, seed: int) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def randn(shape, *, std: float = 1.0, mean: float = 0.0, dtype=torch.bfloat16, device="cpu",
          seed: int = 0) -> torch.Tensor:
    """Seeded normal tensor, drawn in fp32 and rounded to dtype."""
    t = torch.randn(shape, generator=_gen(device, seed), device=device, dtype=torch.float32)
    if std != 1.0:
        t.mul_(std)
    if mean != 0.0:
        t.add_(mean)
    return t.to(dtype)


def rmsnorm_weight(N: int, device="cpu", seed: int = 1) -> torch.Tensor:
    """w = 1 + 0.1 * N(0,1) in bf16."""
    return randn((N,), std=0.1, mean=1.0, device=device, seed=seed)


def embedding_ids(cfg: EmbeddingCfg, device="cpu", seed: int = 2) -> torch.Tensor:
    """int64 [B, S]: 95% uniform over the vocab, 5% from a fixed set of
    `hot_ids` frequent ids (seeded), so duplicates occur."""
    g = torch.Generator(device="cpu")
    g.manual_seed(seed)
    T = cfg.T
    ids = torch.randint(0, cfg.vocab, (T,), generator=g, dtype=torch.int64)
    hot = torch.randint(0, cfg.vocab, (cfg.hot_ids,), generator=g, dtype=torch.int64)
    n_hot = int(round(cfg.hot_frac * T))
    where = torch.randperm(T, generator=g)[:n_hot]
    ids[where] = hot[torch.randint(0, cfg.hot_ids, (n_hot,), generator=g)]
    return ids.view(cfg.batch).to(device)


def rope_positions(cfg: RopeCfg, device="cpu") -> torch.Tensor:
    return torch.arange(cfg.S, dtype=torch.int64, device=device).expand(cfg.B, cfg.S).contiguous()


@dataclass
class Rows:
    """A contiguous row range [lo, hi) of a shared row dimension."""
    lo: int
    hi: int
    meta: dict = field(default_factory=dict)

    @property
    def n(self) -> int:
        return self.hi - self.lo


def shard_rows(total: int, world: int, rank: int) -> Rows:
    """Contiguous split of `total` rows over `world` ranks; the first
    total % world ranks get one extra row."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} for world {world}")
    base, rem = divmod(total, world)
    lo = rank * base + min(rank, rem)
    hi = lo + base + (1 if rank < rem else 0)
    return Rows(lo, hi)
