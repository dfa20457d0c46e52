"""Seeded synthetic paged-decode workloads (the five BASELINE configurations).

Block tables, context lengths and page pools come from numpy's PCG64 generator
(``numpy.random.default_rng(seed)``), so they are bit-identical on every host.
Q/K/V values are N(0, 1) scaled by ``value_std``: drawn with numpy on the host
for the sizes the CPU oracle checks, or with torch's CUDA generator on the
device for the full-size benchmark pools (``values_torch``).

Layout (the reference ABI, include/operator_api.h): q/out [B][Hq][D]; each
cache pool [num_blocks][Hkv][block_size][D]; block_tables [B][max_blocks]
int32 with -1 past each sequence's last page (never read).

Head sharding (``world_size`` > 1): rank r owns KV heads
[r*Hkv/P, (r+1)*Hkv/P) and their query heads, with its own page pool and its
own seeded page shuffle; context lengths are shared by all ranks.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import List, Optional, Sequence, Tuple

import numpy as np

PAGE = 16


@dataclass
class PagedBatch:
    name: str
    num_seqs: int
    num_heads: int          # query heads held by this rank
    num_kv_heads: int       # KV heads held by this rank
    head_size: int
    block_size: int
    dtype: str              # "f16" or "f32" (q, caches and out alike)
    seq_lens: np.ndarray    # int32 [B]
    block_tables: np.ndarray  # int32 [B, max_blocks]
    num_blocks: int         # pages in this rank's pool
    value_std: float
    seed: int
    scale: float
    world_size: int = 1
    rank: int = 0
    total_heads: int = 0    # query heads across all ranks
    notes: dict = field(default_factory=dict)
    kv_elem_size: int = 0   # bytes per K/V element when the cache is quantised (0: elem_size)
    # shared radix prefixes: (member sequence ids, shared leading pages) per group
    prefix_groups: list = field(default_factory=list)

    @property
    def group(self) -> int:
        return self.num_heads // self.num_kv_heads

    @property
    def max_blocks(self) -> int:
        return int(self.block_tables.shape[1])

    @property
    def elem_size(self) -> int:
        return 2 if self.dtype == "f16" else 4

    @property
    def dtype_size(self) -> int:
        return self.elem_size

    @property
    def kv_block_stride(self) -> int:
        return self.num_kv_heads * self.block_size * self.head_size

    @property
    def kv_head_stride(self) -> int:
        return self.block_size * self.head_size

    def pages_per_seq(self) -> np.ndarray:
        return (self.seq_lens.astype(np.int64) + self.block_size - 1) // self.block_size

    @property
    def kv_es(self) -> int:
        return self.kv_elem_size or self.elem_size

    def kv_bytes(self) -> int:
        """K+V bytes the attention reads, counted per sequence (logical)."""
        return int(self.seq_lens.astype(np.int64).sum()) * self.num_kv_heads * \
            self.head_size * 2 * self.kv_es

    def kv_bytes_unique(self) -> int:
        """K+V bytes of distinct (page, slot) cells read: shared prefix pages count once."""
        used = {}
        for b in range(self.num_seqs):
            L = int(self.seq_lens[b])
            npg = (L + self.block_size - 1) // self.block_size
            for j in range(npg):
                phys = int(self.block_tables[b, j])
                n = min(self.block_size, L - j * self.block_size)
                if used.get(phys, 0) < n:
                    used[phys] = n
        return sum(used.values()) * self.num_kv_heads * self.head_size * 2 * self.kv_es

    def algorithmic_bytes(self, unique: bool = False) -> int:
        """KV bytes + Q + out + block-table entries read + seq_lens."""
        kv = self.kv_bytes_unique() if unique else self.kv_bytes()
        qo = 2 * self.num_seqs * self.num_heads * self.head_size * self.elem_size
        bt = int(self.pages_per_seq().sum()) * 4
        return kv + qo + bt + 4 * self.num_seqs

    def flops(self) -> int:
        return int(self.seq_lens.astype(np.int64).sum()) * self.num_heads * 4 * self.head_size

    def context_tokens(self) -> int:
        return int(self.seq_lens.astype(np.int64).sum())

    # ── values ──────────────────────────────────────────────────────────
    def shapes(self) -> Tuple[tuple, tuple]:
        q = (self.num_seqs, self.num_heads, self.head_size)
        kv = (self.num_blocks, self.num_kv_heads, self.block_size, self.head_size)
        return q, kv

    def values_numpy(self) -> Tuple[np.ndarray, np.ndarray, np.ndarray]:
        """Q, K pool, V pool drawn on the host (PCG64, stream [seed, 7, rank])."""
        rng = np.random.default_rng([self.seed, 7, self.rank])
        qs, kvs = self.shapes()
        npd = np.float16 if self.dtype == "f16" else np.float32
        out = []
        for shape in (qs, kvs, kvs):
            x = rng.standard_normal(size=shape, dtype=np.float32) * np.float32(self.value_std)
            out.append(x.astype(npd))
        return tuple(out)

    def values_torch(self, device):
        """Q, K pool, V pool drawn on `device` with torch's generator (seed+rank)."""
        import torch
        g = torch.Generator(device=device)
        g.manual_seed(self.seed * 1000003 + self.rank)
        td = torch.float16 if self.dtype == "f16" else torch.float32
        qs, kvs = self.shapes()
        out = []
        for shape in (qs, kvs, kvs):
            x = torch.empty(shape, dtype=td, device=device)
            # draw in chunks to bound the fp32 temporary
            flat = x.view(-1)
            step = 1 << 27
            for i in range(0, flat.numel(), step):
                n = min(step, flat.numel() - i)
                flat[i:i + n] = (torch.randn(n, generator=g, device=device,
                                             dtype=torch.float32) * self.value_std).to(td)
            out.append(x)
        return tuple(out)

    def values_torch_fp8(self, device, fmt: str = "e4m3"):
        """Q (fp16) and K, V pools quantised to one byte per element (fp8
        "e4m3" / "e5m2", or "int8") with one scale per pool (max |x| maps to
        the format's largest value): (q, k8, v8, k_scale, v_scale), the pools
        as uint8 tensors holding encode(x / scale)."""
        import torch
        q, k, v = self.values_torch(device)
        tdt, fmax = {"e4m3": (torch.float8_e4m3fn, 448.0), "e5m2": (torch.float8_e5m2, 57344.0),
                     "int8": (torch.int8, 127.0)}[fmt]

        def enc(x):  # fp32 -> codes; int8 rounds half to even and saturates
            if tdt is torch.int8:
                return torch.nan_to_num(x, nan=0.0).round().clamp(-128, 127).to(torch.int8)
            return x.to(tdt)
        out = [q]
        scales = []
        for pool in (k, v):
            sc = float(pool.abs().max().float()) / fmax
            flat = pool.view(-1)
            q8 = torch.empty(pool.shape, dtype=torch.uint8, device=device)
            q8f = q8.view(-1)
            step = 1 << 27
            for i in range(0, flat.numel(), step):  # chunks bound the fp32 temporary
                q8f[i:i + step] = enc(flat[i:i + step].float() / sc).view(torch.uint8)
            out.append(q8)
            scales.append(sc)
            del pool
        self.kv_elem_size = 1
        self.notes.update(kv_format=fmt, k_scale=scales[0], v_scale=scales[1])
        return out[0], out[1], out[2], scales[0], scales[1]

    def tables_torch(self, device):
        import torch
        return (torch.from_numpy(np.ascontiguousarray(self.block_tables)).to(device),
                torch.from_numpy(np.ascontiguousarray(self.seq_lens)).to(device))


def _assign_pages(rng: np.random.Generator, lens: Sequence[int], block_size: int,
                  max_blocks: int, slack: float, prefix: Optional[List[int]] = None,
                  prefix_of: Optional[Sequence[int]] = None) -> Tuple[np.ndarray, int]:
    """Block tables over one shuffled pool: shared prefix page sets first (if
    any), then every sequence's private pages as disjoint consecutive slices.
    prefix_of[b] is the index of b's shared prefix in `prefix`, or -1."""
    B = len(lens)
    prefix = prefix or []
    prefix_pages = [p // block_size for p in prefix]
    priv = []
    for b in range(B):
        npg = (int(lens[b]) + block_size - 1) // block_size
        shared = prefix_pages[prefix_of[b]] if prefix_of is not None and prefix_of[b] >= 0 else 0
        priv.append(npg - shared)
    used = sum(prefix_pages) + sum(priv)
    pool = max(1, int(math.ceil(used * (1.0 + slack))))
    perm = rng.permutation(pool).astype(np.int32)
    tables = np.full((B, max_blocks), -1, dtype=np.int32)
    cur = 0
    prefix_ids = []
    for npg in prefix_pages:
        prefix_ids.append(perm[cur:cur + npg])
        cur += npg
    for b in range(B):
        j = 0
        if prefix_of is not None and prefix_of[b] >= 0:
            ids = prefix_ids[prefix_of[b]]
            tables[b, :len(ids)] = ids
            j = len(ids)
        tables[b, j:j + priv[b]] = perm[cur:cur + priv[b]]
        cur += priv[b]
    return tables, pool


def _shard_heads(Hq: int, Hkv: int, world_size: int, rank: int) -> Tuple[int, int]:
    if Hkv % world_size:
        raise ValueError(f"{Hkv} KV heads do not split over {world_size} ranks")
    return Hq // world_size, Hkv // world_size


def make_batch(name: str, lens: Sequence[int], num_heads: int, num_kv_heads: int,
               head_size: int, dtype: str, seed: int, *, block_size: int = PAGE,
               max_blocks: Optional[int] = None, slack: float = 0.1, value_std: float = 1.0,
               world_size: int = 1, rank: int = 0, prefix: Optional[List[int]] = None,
               prefix_of: Optional[Sequence[int]] = None, table_seed: Optional[int] = None
               ) -> PagedBatch:
    lens = np.asarray(lens, dtype=np.int32)
    hq, hkv = _shard_heads(num_heads, num_kv_heads, world_size, rank)
    if max_blocks is None:
        max_blocks = max(1, int((int(lens.max(initial=0)) + block_size - 1) // block_size))
    ts = seed if table_seed is None else table_seed
    rng = np.random.default_rng([ts, 11, rank])
    tables, pool = _assign_pages(rng, lens, block_size, max_blocks, slack, prefix, prefix_of)
    groups = []
    if prefix and prefix_of is not None:
        for gi, plen in enumerate(prefix):
            seqs = [b for b in range(len(lens)) if prefix_of[b] == gi]
            if seqs:
                groups.append((seqs, plen // block_size))
    return PagedBatch(name=name, num_seqs=len(lens), num_heads=hq, num_kv_heads=hkv,
                      head_size=head_size, block_size=block_size, dtype=dtype, seq_lens=lens,
                      block_tables=tables, num_blocks=pool, value_std=value_std, seed=seed,
                      scale=1.0 / math.sqrt(head_size), world_size=world_size, rank=rank,
                      total_heads=num_heads, prefix_groups=groups)


def config1(seed: int = 1) -> PagedBatch:
    """GPT-2-small-shaped, fp32, MHA: B=4, 12/12 heads, D=64, L={37,128,255,512};
    one seeded permutation of a 256-page pool handed out in disjoint slices."""
    lens = np.array([37, 128, 255, 512], dtype=np.int32)
    rng = np.random.default_rng([seed, 11, 0])
    perm = rng.permutation(256).astype(np.int32)
    tables = np.full((4, 32), -1, dtype=np.int32)
    cur = 0
    for b, L in enumerate(lens):
        n = (int(L) + 15) // 16
        tables[b, :n] = perm[cur:cur + n]
        cur += n
    return PagedBatch(name="c1_gpt2_small_fp32", num_seqs=4, num_heads=12, num_kv_heads=12,
                      head_size=64, block_size=16, dtype="f32", seq_lens=lens,
                      block_tables=tables, num_blocks=256, value_std=1.0, seed=seed,
                      scale=1.0 / 8.0, total_heads=12)


def config2(seed: int = 2, num_seqs: int = 64, world_size: int = 1, rank: int = 0) -> PagedBatch:
    """Llama-3-8B GQA: 32/8 heads, D=128, fp16, L~U{1024..8192}, values 0.5*N(0,1),
    pool = total pages + 10 %. With world_size > 1 the KV heads are sharded."""
    rng = np.random.default_rng([seed, 3])
    lens = rng.integers(1024, 8192, size=num_seqs, endpoint=True).astype(np.int32)
    return make_batch("c2_llama3_8b_gqa", lens, 32, 8, 128, "f16", seed, max_blocks=512,
                      value_std=0.5, world_size=world_size, rank=rank)


def config3(seed: int = 3, num_seqs: int = 8) -> PagedBatch:
    """Llama-3-70B long context: 64/8 heads, D=128, fp16, L~U{32768..131072}, N(0,1)."""
    rng = np.random.default_rng([seed, 3])
    lens = rng.integers(32768, 131072, size=num_seqs, endpoint=True).astype(np.int32)
    return make_batch("c3_llama3_70b_long", lens, 64, 8, 128, "f16", seed, max_blocks=8192,
                      value_std=1.0)


def config4(seed: int = 4, num_seqs: int = 256) -> PagedBatch:
    """Prefix sharing: 32/8 heads, D=128, fp16; seqs 0..127 share a 2048-token
    prefix, seqs 128..255 a 512-token one; private suffix U{0..1024} tokens."""
    rng = np.random.default_rng([seed, 3])
    half = num_seqs // 2
    suffix = rng.integers(0, 1024, size=num_seqs, endpoint=True)
    prefix_of = [0] * half + [1] * (num_seqs - half)
    lens = np.array([(2048 if prefix_of[b] == 0 else 512) + int(suffix[b])
                     for b in range(num_seqs)], dtype=np.int32)
    return make_batch("c4_prefix_shared", lens, 32, 8, 128, "f16", seed, max_blocks=192,
                      value_std=0.5, prefix=[2048, 512], prefix_of=prefix_of)


def config5(seed: int = 5, world_size: int = 1, rank: int = 0, num_seqs: int = 512) -> PagedBatch:
    """70B head-sharded scale-out: 64/8 heads, D=128, fp16, B=512,
    L~U{4096..16384}, N(0,1); rank r holds KV heads [r*8/P, (r+1)*8/P)."""
    rng = np.random.default_rng([seed, 3])
    lens = rng.integers(4096, 16384, size=num_seqs, endpoint=True).astype(np.int32)
    return make_batch("c5_llama3_70b_sharded", lens, 64, 8, 128, "f16", seed, max_blocks=1024,
                      value_std=1.0, world_size=world_size, rank=rank)


CONFIGS = {"c1": config1, "c2": config2, "c3": config3, "c4": config4, "c5": config5}
