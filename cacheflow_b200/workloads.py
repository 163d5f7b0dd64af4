"""Seeded synthetic decode workloads with the shapes of the benchmark configs.

Each workload is a batch of sequences over one paged KV pool in CacheFlow's
layout: context lengths, block tables (physical ids drawn from a shuffled
pool), the slot of each sequence's newest token, and the element type.  Cache
contents are generated separately (on the device for benchmarks, on the host
for parity tests) from the same seed.

Named workloads:
  cpu_decode_fp32          8 seqs, ctx U[16,512], 32/32 heads, D 128, fp32 N(0,1),
                           pool = random permutation of 512 blocks
  llama2_7b_ragged_decode  64 seqs, ctx U[128,4096], 32/32 heads, D 128, fp16 N(0,0.5),
                           pool 1.2x the blocks in use, shuffled ids
  llama3_8b_long_decode    16 seqs, ctx log-uniform [16K,128K], 32 q / 8 kv heads,
                           D 128, bf16 N(0,0.5), v2 with 512-token partitions
  continuous_batching_mixed 224 decode rows ctx U[256,8192] + 32 prefill chunks of
                           512 tokens (one causal row per token), half the
                           sequences share a 1024-token prefix (64 shared blocks),
                           16 COW forks, 32 q / 8 kv heads, bf16
  llama3_70b_sharded       1024 seqs, ctx U[512,32768], 64 q / 8 kv heads, bf16,
                           sequences dealt to per-GPU pools
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np

BLOCK = 16


@dataclass
class Workload:
    name: str
    num_heads: int
    num_kv_heads: int
    head_dim: int
    dtype: str  # "f32" | "f16" | "bf16"
    std: float
    context_lens: np.ndarray  # int32 [S]
    block_tables: np.ndarray  # int32 [S, max_blocks_per_seq]
    num_blocks: int  # pool size
    slot_mapping: np.ndarray  # int32 [T] slots of the new tokens written this step
    slot_rows: np.ndarray  # int32 [T] the row (sequence) each new token belongs to
    attention: str = "v1"  # "v1" | "v2"
    copy_pairs: np.ndarray = field(default_factory=lambda: np.zeros((0, 2), np.int64))
    seed: int = 0
    # chunked prefill: rows [num_decode, num_seqs) are the query tokens of the
    # chunks described below (None when the batch is decode rows only)
    num_decode: int | None = None
    chunk_context_lens: np.ndarray | None = None
    chunk_block_tables: np.ndarray | None = None
    chunk_query_start: np.ndarray | None = None

    @property
    def num_seqs(self) -> int:
        return int(self.context_lens.shape[0])

    @property
    def max_context_len(self) -> int:
        return int(self.context_lens.max()) if self.num_seqs else 0

    @property
    def elem_bytes(self) -> int:
        return 4 if self.dtype == "f32" else 2

    def kv_bytes(self) -> int:
        """Algorithmic KV bytes one attention pass reads: each (token, kv head) K and V row once."""
        return int(self.context_lens.astype(np.int64).sum()) * 2 * self.num_kv_heads * self.head_dim * self.elem_bytes

    @property
    def has_chunks(self) -> bool:
        return self.num_decode is not None

    def chunked_kv_bytes(self) -> int:
        """KV bytes of one pass with the prefill rows run as chunks: decode rows
        read their context once, each chunk reads its context once."""
        row = 2 * self.num_kv_heads * self.head_dim * self.elem_bytes
        dec = int(self.context_lens[: self.num_decode].astype(np.int64).sum())
        return (dec + int(self.chunk_context_lens.astype(np.int64).sum())) * row

    def unique_kv_bytes(self) -> int:
        """KV bytes of the distinct physical blocks the batch touches (shared prefixes once)."""
        ids = set()
        for s in range(self.num_seqs):
            n = (int(self.context_lens[s]) + BLOCK - 1) // BLOCK
            ids.update(self.block_tables[s, :n].tolist())
        return len(ids) * BLOCK * 2 * self.num_kv_heads * self.head_dim * self.elem_bytes

    def qo_bytes(self) -> int:
        return 2 * self.num_seqs * self.num_heads * self.head_dim * self.elem_bytes

    def table_bytes(self) -> int:
        return int(((self.context_lens.astype(np.int64) + BLOCK - 1) // BLOCK).sum()) * 4

    def cache_shape(self) -> tuple[int, int, int, int]:
        return (self.num_blocks, self.num_kv_heads, BLOCK, self.head_dim)

    def rehome(self, rows, pool_factor: float = 1.2, seed: int = 0) -> "Workload":
        """Rows `rows` moved into a pool of their own (one GPU's share of a
        sequence-sharded batch): blocks renumbered into a fresh pool of
        pool_factor x the blocks they use, ids shuffled; shared blocks stay
        shared."""
        rows = np.asarray(rows)
        rng = np.random.default_rng(seed)
        ctx = self.context_lens[rows]
        nblk = (ctx.astype(np.int64) + BLOCK - 1) // BLOCK
        old_ids = []
        for i, r in enumerate(rows):
            old_ids.extend(int(b) for b in self.block_tables[r, : nblk[i]])
        uniq = list(dict.fromkeys(old_ids))
        pool = max(1, int(math.ceil(pool_factor * len(uniq))))
        new = rng.permutation(pool)[: len(uniq)]
        remap = dict(zip(uniq, new.tolist()))
        tables = np.zeros((len(rows), max(1, int(nblk.max()) if len(rows) else 1)), np.int32)
        for i, r in enumerate(rows):
            tables[i, : nblk[i]] = [remap[int(b)] for b in self.block_tables[r, : nblk[i]]]
        keep = np.isin(self.slot_rows, rows)
        pos = {int(r): i for i, r in enumerate(rows)}
        new_rows = np.array([pos[int(r)] for r in self.slot_rows[keep]], np.int32)
        slots = np.array([tables[i, (ctx[i] - 1) // BLOCK] * BLOCK + (ctx[i] - 1) % BLOCK for i in new_rows],
                         np.int32).reshape(-1)
        w = Workload(self.name, self.num_heads, self.num_kv_heads, self.head_dim, self.dtype, self.std,
                     ctx.astype(np.int32), tables, pool, slots, new_rows, self.attention, seed=self.seed)
        return w

    def subset(self, rows: np.ndarray) -> "Workload":
        """Same pool, only the given rows (for oracle checks of large batches)."""
        rows = np.asarray(rows)
        keep = np.isin(self.slot_rows, rows)
        remap = {int(r): i for i, r in enumerate(rows)}
        return Workload(self.name + "[subset]", self.num_heads, self.num_kv_heads, self.head_dim,
                        self.dtype, self.std, self.context_lens[rows].copy(),
                        self.block_tables[rows].copy(), self.num_blocks,
                        self.slot_mapping[keep].copy(),
                        np.array([remap[int(r)] for r in self.slot_rows[keep]], np.int32),
                        self.attention, self.copy_pairs, self.seed)


def _tables(rng, ctx: np.ndarray, pool: int, ids: np.ndarray | None = None):
    nblk = (ctx.astype(np.int64) + BLOCK - 1) // BLOCK
    total = int(nblk.sum())
    if ids is None:
        ids = rng.permutation(pool)[:total]
    mbps = max(1, int(nblk.max()))
    tables = np.zeros((ctx.shape[0], mbps), np.int32)
    off = 0
    for s, n in enumerate(nblk):
        tables[s, :n] = ids[off:off + n]
        off += n
    return tables


def _last_slots(ctx: np.ndarray, tables: np.ndarray) -> np.ndarray:
    pos = ctx.astype(np.int64) - 1
    return (tables[np.arange(ctx.shape[0]), pos // BLOCK].astype(np.int64) * BLOCK + pos % BLOCK).astype(np.int32)


def decode_batch(name, ctx, num_heads, num_kv_heads, head_dim, dtype, std, seed, pool=None,
                 pool_factor=1.2, attention="v1") -> Workload:
    rng = np.random.default_rng(seed + 1)
    ctx = np.asarray(ctx, np.int32)
    total = int(((ctx.astype(np.int64) + BLOCK - 1) // BLOCK).sum())
    if pool is None:
        pool = int(math.ceil(pool_factor * total))
    tables = _tables(rng, ctx, pool)
    slots = _last_slots(ctx, tables)
    return Workload(name, num_heads, num_kv_heads, head_dim, dtype, std, ctx, tables, pool, slots,
                    np.arange(ctx.shape[0], dtype=np.int32), attention, seed=seed)


def cpu_decode_fp32(seed: int = 1234) -> Workload:
    rng = np.random.default_rng(seed)
    ctx = rng.integers(16, 513, 8)
    return decode_batch("cpu_decode_fp32", ctx, 32, 32, 128, "f32", 1.0, seed, pool=512)


def llama2_7b_ragged_decode(seed: int = 1234, num_seqs: int = 64) -> Workload:
    rng = np.random.default_rng(seed)
    ctx = rng.integers(128, 4097, num_seqs)
    return decode_batch("llama2_7b_ragged_decode", ctx, 32, 32, 128, "f16", 0.5, seed)


def llama3_8b_long_decode(seed: int = 1234, num_seqs: int = 16) -> Workload:
    rng = np.random.default_rng(seed)
    ctx = np.exp(rng.uniform(math.log(16384), math.log(131072), num_seqs)).astype(np.int64)
    return decode_batch("llama3_8b_long_decode", ctx, 32, 8, 128, "bf16", 0.5, seed, attention="v2")


def llama3_70b_sharded(seed: int = 1234, num_seqs: int = 1024) -> Workload:
    rng = np.random.default_rng(seed)
    ctx = rng.integers(512, 32769, num_seqs)
    return decode_batch("llama3_70b_sharded", ctx, 64, 8, 128, "bf16", 0.5, seed, attention="v2")


def continuous_batching_mixed(seed: int = 1234) -> Workload:
    """224 decode rows + 32 prefill chunks of 512 tokens as causal per-token rows.

    Half of the 256 sequences start with the same 1024-token prefix (64 shared
    block ids).  16 decode sequences that share the prefix fork: their last
    block is copied (COW) to a fresh block before the new token is written.
    """
    rng = np.random.default_rng(seed)
    n_dec, n_pre, chunk, prefix = 224, 32, 512, 1024
    dec_ctx = rng.integers(256, 8193, n_dec)
    pre_start = rng.integers(0, 4097, n_pre) // BLOCK * BLOCK  # tokens already cached
    shared = np.zeros(n_dec + n_pre, bool)
    shared[rng.permutation(n_dec + n_pre)[: (n_dec + n_pre) // 2]] = True
    pre_total = pre_start + chunk
    seq_len = np.concatenate([dec_ctx, pre_total]).astype(np.int64)
    # New tokens never land in the shared prefix: a decode row needs at least
    # one own token past it, a prefill chunk starts at or after it.
    is_pre = np.arange(n_dec + n_pre) >= n_dec
    seq_len[shared & ~is_pre] = np.maximum(seq_len[shared & ~is_pre], prefix + 1)
    seq_len[shared & is_pre] = np.maximum(seq_len[shared & is_pre], prefix + chunk)
    nblk = (seq_len + BLOCK - 1) // BLOCK
    n_shared_blk = prefix // BLOCK
    own = nblk - np.where(shared, n_shared_blk, 0)
    n_forks = 16
    total = int(own.sum()) + n_shared_blk + n_forks
    pool = int(math.ceil(1.2 * total))
    ids = rng.permutation(pool)
    shared_ids, ids = ids[:n_shared_blk], ids[n_shared_blk:]
    mbps = int(nblk.max())
    seq_tables = np.zeros((n_dec + n_pre, mbps), np.int32)
    off = 0
    for s in range(n_dec + n_pre):
        k = 0
        if shared[s]:
            seq_tables[s, :n_shared_blk] = shared_ids
            k = n_shared_blk
        n = int(own[s])
        seq_tables[s, k:k + n] = ids[off:off + n]
        off += n
    # COW forks: decode sequences sharing the prefix whose new token lands in a
    # shared block get a private copy of that block.
    fork_src, fork_dst = [], []
    cand = [s for s in range(n_dec) if shared[s]]
    for s in rng.permutation(cand)[:n_forks]:
        b = int(rng.integers(0, n_shared_blk))
        fork_src.append(int(seq_tables[s, b]))
        fork_dst.append(int(ids[off]))
        seq_tables[s, b] = ids[off]
        off += 1
    # Rows: decode rows (one query each), then per prefill sequence one row per
    # chunk token with causal context length.
    rows_ctx = [int(x) for x in seq_len[:n_dec]]
    rows_tab = [seq_tables[s] for s in range(n_dec)]
    slots, slot_rows = [], []
    for s in range(n_dec):
        pos = rows_ctx[s] - 1
        slots.append(int(seq_tables[s, pos // BLOCK]) * BLOCK + pos % BLOCK)
        slot_rows.append(s)
    for i in range(n_pre):
        s = n_dec + i
        start = int(seq_len[s]) - chunk
        for t in range(chunk):
            pos = start + t
            r = len(rows_ctx)
            rows_ctx.append(pos + 1)
            rows_tab.append(seq_tables[s])
            slots.append(int(seq_tables[s, pos // BLOCK]) * BLOCK + pos % BLOCK)
            slot_rows.append(r)
    ctx = np.array(rows_ctx, np.int32)
    tables = np.stack(rows_tab).astype(np.int32)
    w = Workload("continuous_batching_mixed", 32, 8, 128, "bf16", 0.5, ctx, tables, pool,
                 np.array(slots, np.int32), np.array(slot_rows, np.int32), "v1", seed=seed)
    w.copy_pairs = np.stack([np.array(fork_src, np.int64), np.array(fork_dst, np.int64)], 1)
    # The same prefill work as chunks for the multi-query operator: rows
    # n_dec.. are the chunks' tokens, chunk-major.
    w.num_decode = n_dec
    w.chunk_context_lens = seq_len[n_dec:].astype(np.int32)
    w.chunk_block_tables = seq_tables[n_dec:].astype(np.int32)
    w.chunk_query_start = (np.arange(n_pre + 1) * chunk).astype(np.int32)
    return w


WORKLOADS = {
    "cpu_decode_fp32": cpu_decode_fp32,
    "llama2_7b_ragged_decode": llama2_7b_ragged_decode,
    "llama3_8b_long_decode": llama3_8b_long_decode,
    "continuous_batching_mixed": continuous_batching_mixed,
    "llama3_70b_sharded": llama3_70b_sharded,
}


def make(name: str, **kw) -> Workload:
    return WORKLOADS[name](**kw)


# ---------------------------------------------------------------------------
# Device-resident state of a workload (seeded, generated on the GPU).
# ---------------------------------------------------------------------------
TORCH_DTYPES = {"f32": "float32", "f16": "float16", "bf16": "bfloat16"}


def device_state(w: Workload, device, seed: int = 4321) -> dict:
    """Caches, query, new K/V rows and index tensors of `w` on `device`."""
    import torch

    dt = getattr(torch, TORCH_DTYPES[w.dtype])
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    S, H, Hkv, D = w.num_seqs, w.num_heads, w.num_kv_heads, w.head_dim
    T = len(w.slot_mapping)
    st = {
        "k_cache": torch.empty(w.cache_shape(), dtype=dt, device=device).normal_(0, w.std, generator=gen),
        "v_cache": torch.empty(w.cache_shape(), dtype=dt, device=device).normal_(0, w.std, generator=gen),
        "q": torch.empty((S, H, D), dtype=dt, device=device).normal_(0, w.std, generator=gen),
        "k_new": torch.empty((T, Hkv, D), dtype=dt, device=device).normal_(0, w.std, generator=gen),
        "v_new": torch.empty((T, Hkv, D), dtype=dt, device=device).normal_(0, w.std, generator=gen),
        "slots": torch.from_numpy(w.slot_mapping).to(device),
        "tables": torch.from_numpy(w.block_tables).to(device),
        "ctx": torch.from_numpy(w.context_lens).to(device),
        "pairs": torch.from_numpy(w.copy_pairs).to(device) if len(w.copy_pairs) else None,
    }
    return st


def gather_rows_for_oracle(w: Workload, st: dict, rows) -> tuple:
    """Host copies of what rows `rows` of the batch read, with their blocks
    renumbered into a compact pool: (q, k, v, tables, context_lens) as numpy
    (bf16 as uint16 bits), small enough for the CPU oracle."""
    import torch

    rows = np.asarray(rows)
    ctx = w.context_lens[rows]
    nblk = (ctx.astype(np.int64) + BLOCK - 1) // BLOCK
    used = []
    remap = {}
    tables = np.zeros((len(rows), int(nblk.max())), np.int32)
    for i, r in enumerate(rows):
        for b in range(nblk[i]):
            old = int(w.block_tables[r, b])
            if old not in remap:
                remap[old] = len(used)
                used.append(old)
            tables[i, b] = remap[old]
    idx = torch.tensor(used, dtype=torch.int64, device=st["k_cache"].device)
    ridx = torch.from_numpy(rows.astype(np.int64)).to(st["q"].device)

    def host(t):
        t = t.contiguous().cpu()
        if t.dtype == torch.bfloat16:
            return t.view(torch.int16).numpy().view(np.uint16)
        return t.numpy()

    return (host(st["q"].index_select(0, ridx)), host(st["k_cache"].index_select(0, idx)),
            host(st["v_cache"].index_select(0, idx)), tables, ctx.astype(np.int32))


# ---------------------------------------------------------------------------
# Host-side tensors for parity checks (numpy; bf16 as uint16 bit patterns).
# ---------------------------------------------------------------------------
def host_values(shape, dtype: str, std: float, rng: np.random.Generator) -> np.ndarray:
    x = (rng.standard_normal(shape, dtype=np.float32) * np.float32(std))
    if dtype == "f32":
        return x
    if dtype == "f16":
        return x.astype(np.float16)
    # round-to-nearest-even to bf16, kept as raw bits
    u = x.view(np.uint32)
    r = ((u >> 16) & 1) + np.uint32(0x7FFF)
    return ((u + r) >> 16).astype(np.uint16)
