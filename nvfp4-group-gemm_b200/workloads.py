"""Seeded synthetic NVFP4 grouped-GEMM problems (the benchmark configurations).

No dataset exists for this path; every configuration is synthetic with the
shapes and value distributions the benchmark specification names:

* e2m1 codes uniform over all 16 codes (both nibbles of each byte uniform);
* E4M3 scales 2^U{-4..3} per 16 elements along K (stored plain and blocked);
* per-group fp32 global scale (1.0, or U[0.5, 2] where the configuration says so);
* fp16 outputs prefilled with randn, like the harness (REFERENCE_IMPL.md:187).

``distribution="reference"`` switches to the harness generator's distribution
(REFERENCE_IMPL.md:143-205): nibbles masked with 0b1011 (codes {0, +-0.5, +-1,
+-1.5}) and scales in {1, 2}.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np
import torch

from .layout import blocked_as_reordered, plain_to_blocked

CHALLENGE_SHAPES = {
    # name: (M per group, N, K) -- the reference's speed-of-light shape sets (CHALLENGE.md:53-56)
    "challenge1": ((80, 176, 128, 72, 64, 248, 96, 160), 4096, 7168),
    "challenge2": ((40, 76, 168, 72, 164, 148, 196, 160), 7168, 2048),
    "challenge3": ((192, 320), 3072, 4096),
    "challenge4": ((128, 384), 4096, 1536),
}


@dataclass
class GroupedProblem:
    """A grouped problem with tensors on one device (scales in both layouts)."""

    name: str
    m: list
    n: int
    k: int
    gated: bool
    a: list                      # uint8 [m, k/2]
    b: list                      # uint8 [n, k/2]   (gate weights when gated)
    c: list                      # fp16 [m, n]
    sfa_plain: list              # uint8 [m, k/16]
    sfb_plain: list
    sfa: list                    # blocked uint8 (flat)
    sfb: list
    alpha: list
    b2: list | None = None       # up weights when gated
    sfb2_plain: list | None = None
    sfb2: list | None = None
    alpha2: list | None = None
    meta: dict = field(default_factory=dict)

    @property
    def num_groups(self) -> int:
        return len(self.m)

    def problem_sizes(self) -> list:
        return [(m, self.n, self.k, 1) for m in self.m]

    def flops(self) -> float:
        """Algorithmic FLOPs: 2*M*N*K per product (two products when gated)."""
        return float(sum(2 * m * self.n * self.k for m in self.m)) * (2 if self.gated else 1)

    def algorithmic_bytes(self) -> float:
        """Bytes a perfect kernel moves: packed A and B, E4M3 scales, fp16 C.

        Weights of empty groups are not counted (they are never read).
        """
        tot = 0
        nb = 2 if self.gated else 1
        for m in self.m:
            if m == 0:
                continue
            tot += m * self.k // 2 + m * self.k // 16
            tot += nb * (self.n * self.k // 2 + self.n * self.k // 16)
            tot += m * self.n * 2
        return float(tot)

    def input_bytes(self) -> int:
        """Bytes of the operands as stored (A, B, blocked scales)."""
        ts = self.a + self.b + self.sfa + self.sfb + (self.b2 or []) + (self.sfb2 or [])
        return int(sum(t.numel() * t.element_size() for t in ts))

    def output_bytes(self) -> int:
        return int(sum(t.numel() * t.element_size() for t in self.c))

    def reference_data(self, fp4_dtype: bool = True) -> tuple:
        """The harness-shaped 4-tuple (a/b as [rows, K/2, 1], reordered 6-D scale views)."""
        f4 = getattr(torch, "float4_e2m1fn_x2", None) if fp4_dtype else None

        def op(t):
            v = t.unsqueeze(-1)
            return v.view(f4) if f4 is not None else v

        sfr = []
        abc = []
        plain = []
        for g, m in enumerate(self.m):
            sa = blocked_as_reordered(self.sfa[g], m, self.k)
            sb = blocked_as_reordered(self.sfb[g], self.n, self.k)
            if self.gated:
                sb2 = blocked_as_reordered(self.sfb2[g], self.n, self.k)
                abc.append((op(self.a[g]), op(self.b[g]), op(self.b2[g]), self.c[g].unsqueeze(-1)))
                sfr.append((sa, sb, sb2))
                plain.append((self.sfa_plain[g], self.sfb_plain[g], self.sfb2_plain[g]))
            else:
                abc.append((op(self.a[g]), op(self.b[g]), self.c[g].unsqueeze(-1)))
                sfr.append((sa, sb))
                plain.append((self.sfa_plain[g], self.sfb_plain[g]))
        return (abc, plain, sfr, self.problem_sizes())

    def global_scales(self) -> list:
        if self.gated:
            return [(a, b) for a, b in zip(self.alpha, self.alpha2)]
        return list(self.alpha)


def _e2m1_bytes(gen: torch.Generator, rows: int, kbytes: int, distribution: str,
                device) -> torch.Tensor:
    t = torch.randint(0, 256, (rows, kbytes), dtype=torch.uint8, generator=gen, device=device)
    if distribution == "reference":
        t &= 0b1011_1011
    return t


def _sf_bytes(gen: torch.Generator, rows: int, sf_cols: int, distribution: str,
              device) -> torch.Tensor:
    if distribution == "reference":
        # randint(1, 3) -> E4M3 1.0 (0x38) or 2.0 (0x40)
        e = torch.randint(0, 2, (rows, sf_cols), dtype=torch.int32, generator=gen, device=device)
        t = (0x38 + 8 * e).to(torch.uint8)
    else:
        # 2^e, e uniform in [-4, 3]: E4M3 biased exponent e + 7 in bits 6..3, zero mantissa
        e = torch.randint(-4, 4, (rows, sf_cols), dtype=torch.int32, generator=gen, device=device)
        t = ((e + 7) << 3).to(torch.uint8)
    return t


def make_problem(name: str, m_list, n: int, k: int, *, gated: bool = False, seed: int = 0,
                 device="cuda", distribution: str = "baseline", alpha_range=None,
                 meta: dict | None = None) -> GroupedProblem:
    """Build a grouped problem with seeded inputs, generated directly on `device`.

    The random streams of the CPU and CUDA generators differ, so the same seed
    gives different (equally distributed) values on different device types.
    """
    if k % 256 != 0:
        raise ValueError("K must be a multiple of 256")
    device = torch.device(device)
    gen = torch.Generator(device=device).manual_seed(seed)
    rng = np.random.default_rng(seed)
    G = len(m_list)
    a, b, b2, c = [], [], [], []
    sfa_p, sfb_p, sfb2_p, sfa, sfb, sfb2 = [], [], [], [], [], []
    for g in range(G):
        m = int(m_list[g])
        a.append(_e2m1_bytes(gen, m, k // 2, distribution, device))
        b.append(_e2m1_bytes(gen, n, k // 2, distribution, device))
        sa = _sf_bytes(gen, m, k // 16, distribution, device)
        sb = _sf_bytes(gen, n, k // 16, distribution, device)
        sfa_p.append(sa)
        sfb_p.append(sb)
        sfa.append(plain_to_blocked(sa))
        sfb.append(plain_to_blocked(sb))
        if gated:
            b2.append(_e2m1_bytes(gen, n, k // 2, distribution, device))
            sb2 = _sf_bytes(gen, n, k // 16, distribution, device)
            sfb2_p.append(sb2)
            sfb2.append(plain_to_blocked(sb2))
        c.append(torch.randn((m, n), generator=gen, dtype=torch.float32, device=device)
                 .to(torch.float16))
    if alpha_range is None:
        alpha = [1.0] * G
        alpha2 = [1.0] * G if gated else None
    else:
        lo, hi = alpha_range
        alpha = [float(x) for x in rng.uniform(lo, hi, G).astype(np.float32)]
        alpha2 = [float(x) for x in rng.uniform(lo, hi, G).astype(np.float32)] if gated else None
    return GroupedProblem(name=name, m=[int(x) for x in m_list], n=n, k=k, gated=gated, a=a, b=b,
                          c=c, sfa_plain=sfa_p, sfb_plain=sfb_p, sfa=sfa, sfb=sfb, alpha=alpha,
                          b2=b2 if gated else None, sfb2_plain=sfb2_p if gated else None,
                          sfb2=sfb2 if gated else None, alpha2=alpha2, meta=meta or {})


# ----------------------------------------------------------------------------
# Row counts per expert
# ----------------------------------------------------------------------------
def zipf_topk_rows(num_experts: int, tokens: int, topk: int, s: float, seed: int) -> list:
    """Rows per expert when each token picks `topk` distinct experts with Zipf(s) popularity."""
    rng = np.random.default_rng(seed)
    p = 1.0 / np.arange(1, num_experts + 1, dtype=np.float64) ** s
    p /= p.sum()
    perm = rng.permutation(num_experts)  # popular experts are not the first ids
    counts = np.zeros(num_experts, dtype=np.int64)
    for _ in range(tokens):
        chosen = rng.choice(num_experts, size=topk, replace=False, p=p)
        counts[perm[chosen]] += 1
    return counts.tolist()


def uniform_topk_rows(num_experts: int, tokens: int, topk: int, seed: int) -> list:
    """Rows per expert when each token picks `topk` distinct experts uniformly at random."""
    rng = np.random.default_rng(seed)
    keys = rng.random((tokens, num_experts), dtype=np.float32)
    chosen = np.argpartition(keys, topk, axis=1)[:, :topk]
    return np.bincount(chosen.reshape(-1), minlength=num_experts).tolist()


# ----------------------------------------------------------------------------
# The benchmark configurations
# ----------------------------------------------------------------------------
def config_rows(name: str, seed: int = 0) -> tuple:
    """(m_list, n, k, gated, alpha_range) of a named configuration."""
    if name == "cfg1":
        return [128], 256, 512, False, None
    if name == "cfg2":
        return [1024] * 8, 4096, 7168, False, (0.5, 2.0)
    if name == "cfg3":
        rng = np.random.default_rng(seed)
        return [int(128 * x) for x in rng.integers(2, 17, 8)], 2048, 7168, True, None
    if name == "cfg4":
        return zipf_topk_rows(64, 512, 8, 1.2, seed), 1536, 4096, False, None
    if name == "cfg5":
        return uniform_topk_rows(256, 32768, 8, seed), 2048, 7168, True, None
    if name == "moe_down":
        # cfg5's down projection: the same routed rows, N = hidden 7168, K = intermediate 2048
        return uniform_topk_rows(256, 32768, 8, seed), 7168, 2048, False, None
    if name == "decode":
        # cfg4's experts at a decode step of 64 tokens x top-8: 512 rows over 64 experts
        return zipf_topk_rows(64, 64, 8, 1.2, seed), 1536, 4096, False, None
    if name in CHALLENGE_SHAPES:
        ms, n, k = CHALLENGE_SHAPES[name]
        return list(ms), n, k, False, None
    raise KeyError(f"unknown configuration {name!r}")


def make_config(name: str, seed: int = 0, device="cuda", experts: slice | None = None,
                distribution: str | None = None) -> GroupedProblem:
    """Inputs of a named configuration; `experts` selects a contiguous expert shard."""
    m_list, n, k, gated, alpha_range = config_rows(name, seed)
    if distribution is None:
        distribution = "reference" if name.startswith("challenge") else "baseline"
    meta = {"all_m": list(m_list)}
    if experts is not None:
        meta["experts"] = (experts.start, experts.stop)
        m_list = m_list[experts]
        seed = seed * 1000003 + (experts.start or 0)
    return make_problem(name, m_list, n, k, gated=gated, seed=seed, device=device,
                        distribution=distribution, alpha_range=alpha_range, meta=meta)
