"""Python access to the CPU oracle (cf_oracle.c) and to the reference-derived
libraries under oracle/_ref/.

TEST / BENCH INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke()
and the CPU-baseline leg of bench.py as the oracle.  The product package
(cacheflow_b200) never imports this module.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from ctypes import POINTER, c_double, c_float, c_int32, c_int64, c_void_p
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_LIB = HERE / "libcf_oracle.so"
REF_CUDA_LIB = HERE / "_ref" / "libcf_ref_cuda.so"
REF_CPU_LIB = HERE / "_ref" / "libcf_ref_cpu.so"

DTYPE_CODE = {np.dtype(np.float32): 0, np.dtype(np.float16): 1}
BF16 = 2  # numpy has no bfloat16: bf16 arrays are carried as uint16 bit patterns


REF_API_LIB = HERE / "_ref" / "libcf_ref_api.so"
REF_ENGINE_LIB = HERE / "_ref" / "libcf_ref_engine.so"


def reference_dir() -> Path | None:
    """The CacheFlow checkout: $CF_REFERENCE_DIR, else a `reference` directory
    beside this checkout; None when neither holds src/cacheflow."""
    env = os.environ.get("CF_REFERENCE_DIR")
    cand = Path(env) if env else HERE.parent.parent / "reference"
    return cand if (cand / "src" / "cacheflow").is_dir() else None


def build(with_reference: bool | None = None) -> None:
    """Builds the oracle (and, when the reference checkout exists, oracle/_ref)."""
    subprocess.run(["make", "-s", "-C", str(HERE), "libcf_oracle.so"], check=True)
    ref = reference_dir()
    if with_reference is None:
        with_reference = ref is not None
    if with_reference:
        if ref is None:
            raise RuntimeError("CacheFlow sources not found: set CF_REFERENCE_DIR")
        subprocess.run(["make", "-s", "-C", str(HERE), "ref", f"REF={ref}"], check=True)


_LIB = None


def lib() -> ctypes.CDLL:
    global _LIB
    if _LIB is None:
        if not ORACLE_LIB.exists():
            build(with_reference=False)
        L = ctypes.CDLL(str(ORACLE_LIB))
        L.cfo_paged_attention.argtypes = [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                          c_float] + [c_int32] * 8
        L.cfo_paged_attention_partitions.argtypes = [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                                     c_float] + [c_int32] * 9 + [c_void_p] * 3
        L.cfo_paged_attention_reduce.argtypes = [c_void_p, c_void_p, c_void_p, c_void_p] + [c_int32] * 5 + [c_void_p]
        L.cfo_reshape_and_cache.argtypes = [c_void_p] * 5 + [c_int32] * 5
        L.cfo_copy_blocks.argtypes = [c_void_p, c_void_p, c_void_p, c_int32, c_int64]
        L.cfo_swap_blocks.argtypes = [c_void_p, c_void_p, c_void_p, c_int32, c_int64]
        L.cfo_compact_kv_cache.argtypes = [c_void_p, c_void_p, c_void_p, c_void_p, c_int32, c_int64]
        L.cfo_memset_blocks.argtypes = [c_void_p, c_void_p, c_int32, c_int64]
        L.cfo_paged_attention_fp8.argtypes = [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                              c_float] + [c_int32] * 7 + [c_float, c_float, c_int32]
        L.cfo_e4m3_from_float.restype = ctypes.c_uint8
        L.cfo_e4m3_from_float.argtypes = [c_float]
        L.cfo_reshape_and_cache_fp8.argtypes = [c_void_p] * 5 + [c_int32] * 5 + [c_float, c_float]
        L.cfo_build_decode_inputs.restype = c_int32
        L.cfo_build_decode_inputs.argtypes = [c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_int32,
                                              c_void_p, c_void_p, c_void_p]
        L.cfo_load.restype = c_double
        L.cfo_load.argtypes = [c_void_p, c_int64, c_int32]
        _LIB = L
    return _LIB


def _p(a: np.ndarray) -> int:
    assert a.flags.c_contiguous
    return a.ctypes.data


def _code(a: np.ndarray, dtype_code: int | None) -> int:
    if dtype_code is not None:
        return dtype_code
    return DTYPE_CODE[a.dtype]


def paged_attention(q, k_cache, v_cache, block_tables, context_lens, scale, dtype_code=None,
                    num_threads=1) -> np.ndarray:
    """float64 [S, H, D] attention output (the intended softmax attention)."""
    S, H, D = q.shape
    _, Hkv, bs, _ = k_cache.shape
    out = np.zeros((S, H, D), dtype=np.float64)
    bt = np.ascontiguousarray(block_tables, dtype=np.int32)
    cl = np.ascontiguousarray(context_lens, dtype=np.int32)
    lib().cfo_paged_attention(_p(q), _p(k_cache), _p(v_cache), _p(out), _p(bt), _p(cl), float(scale),
                              S, H, Hkv, D, bs, bt.shape[1], _code(q, dtype_code), num_threads)
    return out


def paged_attention_fp8(q, k_cache, v_cache, block_tables, context_lens, scale, k_scale, v_scale,
                        dtype_code=None, num_threads=1) -> np.ndarray:
    """float64 attention over e4m3 caches (uint8 arrays): K = k_scale * stored, V = v_scale * stored."""
    S, H, D = q.shape
    _, Hkv, bs, _ = k_cache.shape
    assert k_cache.dtype == np.uint8 and v_cache.dtype == np.uint8
    out = np.zeros((S, H, D), dtype=np.float64)
    bt = np.ascontiguousarray(block_tables, dtype=np.int32)
    cl = np.ascontiguousarray(context_lens, dtype=np.int32)
    lib().cfo_paged_attention_fp8(_p(q), _p(k_cache), _p(v_cache), _p(out), _p(bt), _p(cl), float(scale), S, H, Hkv,
                                  D, bs, bt.shape[1], _code(q, dtype_code), float(k_scale), float(v_scale),
                                  num_threads)
    return out


def e4m3_from_float(x) -> np.ndarray:
    """uint8 e4m3 codes of float32 values (nearest, ties to even, saturating at 448)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    f = lib().cfo_e4m3_from_float
    return np.array([f(float(v)) for v in x.reshape(-1)], np.uint8).reshape(x.shape)


def e4m3_to_float(codes) -> np.ndarray:
    c = np.ascontiguousarray(codes, dtype=np.uint8)
    f = lib().cfo_load
    return np.array([f(c.ctypes.data, i, 3) for i in range(c.size)], np.float64).reshape(c.shape)


def reshape_and_cache_fp8(key, value, key_cache, value_cache, slot_mapping, k_scale, v_scale,
                          dtype_code=None) -> None:
    """In place on uint8 key_cache / value_cache."""
    T, Hkv, D = key.shape
    bs = key_cache.shape[2]
    sm = np.ascontiguousarray(slot_mapping, dtype=np.int32)
    lib().cfo_reshape_and_cache_fp8(_p(key), _p(value), _p(key_cache), _p(value_cache), _p(sm), T, Hkv, D, bs,
                                    _code(key, dtype_code), float(k_scale), float(v_scale))


def paged_attention_partitions(q, k_cache, v_cache, block_tables, context_lens, scale,
                               partition_size, num_partitions, dtype_code=None):
    S, H, D = q.shape
    _, Hkv, bs, _ = k_cache.shape
    mx = np.full((S, H, num_partitions), np.nan)
    es = np.full((S, H, num_partitions), np.nan)
    to = np.full((S, H, num_partitions, D), np.nan)
    bt = np.ascontiguousarray(block_tables, dtype=np.int32)
    cl = np.ascontiguousarray(context_lens, dtype=np.int32)
    lib().cfo_paged_attention_partitions(_p(q), _p(k_cache), _p(v_cache), _p(bt), _p(cl), float(scale),
                                         S, H, Hkv, D, bs, bt.shape[1], _code(q, dtype_code),
                                         partition_size, num_partitions, _p(mx), _p(es), _p(to))
    return mx, es, to


def paged_attention_reduce(mx, es, to, context_lens, partition_size) -> np.ndarray:
    S, H, P, D = to.shape
    out = np.zeros((S, H, D))
    cl = np.ascontiguousarray(context_lens, dtype=np.int32)
    lib().cfo_paged_attention_reduce(_p(np.ascontiguousarray(mx)), _p(np.ascontiguousarray(es)),
                                     _p(np.ascontiguousarray(to)), _p(cl), S, H, D, partition_size,
                                     P, _p(out))
    return out


def reshape_and_cache(key, value, key_cache, value_cache, slot_mapping) -> None:
    """In place on key_cache / value_cache (numpy, any dtype)."""
    T, Hkv, D = key.shape
    bs = key_cache.shape[2]
    sm = np.ascontiguousarray(slot_mapping, dtype=np.int32)
    lib().cfo_reshape_and_cache(_p(key), _p(value), _p(key_cache), _p(value_cache), _p(sm), T, Hkv, D,
                                bs, key.itemsize)


def copy_blocks(key_cache, value_cache, block_mapping) -> None:
    m = np.ascontiguousarray(block_mapping, dtype=np.int64)
    lib().cfo_copy_blocks(_p(key_cache), _p(value_cache), _p(m), m.shape[0],
                          key_cache[0].nbytes)


def swap_blocks(src, dst, block_mapping) -> None:
    m = np.ascontiguousarray(block_mapping, dtype=np.int64)
    lib().cfo_swap_blocks(_p(src), _p(dst), _p(m), m.shape[0], src[0].nbytes)


def compact_kv_cache(key_cache, value_cache, src_ids, dst_ids) -> None:
    s = np.ascontiguousarray(src_ids, dtype=np.int32)
    d = np.ascontiguousarray(dst_ids, dtype=np.int32)
    lib().cfo_compact_kv_cache(_p(key_cache), _p(value_cache), _p(s), _p(d), s.shape[0],
                               key_cache[0].nbytes)


def memset_blocks(cache, block_ids) -> None:
    b = np.ascontiguousarray(block_ids, dtype=np.int32)
    lib().cfo_memset_blocks(_p(cache), _p(b), b.shape[0], cache[0].nbytes)


def build_decode_inputs(positions, block_offsets, block_ids, max_blocks_per_seq, block_size=16):
    """(block_tables, context_lens, slot_mapping, rows cut) of prepare_kv_cache_inputs."""
    pos = np.ascontiguousarray(positions, dtype=np.int32)
    off = np.ascontiguousarray(block_offsets, dtype=np.int64)
    ids = np.ascontiguousarray(block_ids, dtype=np.int32)
    if ids.size == 0:
        ids = np.zeros(1, np.int32)
    S = pos.shape[0]
    tables = np.zeros((S, max_blocks_per_seq), np.int32)
    ctx = np.zeros(S, np.int32)
    slots = np.zeros(S, np.int32)
    cut = lib().cfo_build_decode_inputs(_p(pos), _p(off), _p(ids), S, max_blocks_per_seq, block_size,
                                        _p(tables), _p(ctx), _p(slots))
    return tables, ctx, slots, int(cut)


# ---------------------------------------------------------------------------
# numpy restatement of the attention math (independent second restatement,
# used to cross-check the C oracle on small cases).
# ---------------------------------------------------------------------------
def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << 16).view(np.float32)


def to_f64(a: np.ndarray, dtype_code: int | None = None) -> np.ndarray:
    if dtype_code == BF16:
        return bf16_bits_to_f32(a).astype(np.float64)
    return a.astype(np.float64)


def paged_attention_numpy(q, k_cache, v_cache, block_tables, context_lens, scale, dtype_code=None):
    qd, kd, vd = (to_f64(x, dtype_code) for x in (q, k_cache, v_cache))
    S, H, D = q.shape
    Hkv, bs = k_cache.shape[1], k_cache.shape[2]
    out = np.zeros((S, H, D))
    for s in range(S):
        ctx = int(context_lens[s])
        if ctx == 0:
            continue
        t = np.arange(ctx)
        phys = np.asarray(block_tables[s])[t // bs]
        for h in range(H):
            kvh = h // (H // Hkv)
            K = kd[phys, kvh, t % bs]
            V = vd[phys, kvh, t % bs]
            sc = (K @ qd[s, h]) * np.float64(np.float32(scale))
            w = np.exp(sc - sc.max())
            out[s, h] = (w @ V) / w.sum()
    return out


# ---------------------------------------------------------------------------
# Reference-derived libraries (built from the reference sources by Makefile).
# ---------------------------------------------------------------------------
class RefCuda:
    """CacheFlow's own CUDA kernels (fp32), for GPU-side comparison."""

    def __init__(self):
        if not REF_CUDA_LIB.exists():
            raise FileNotFoundError(f"{REF_CUDA_LIB} not built (make -C oracle ref)")
        L = ctypes.CDLL(str(REF_CUDA_LIB), mode=os.RTLD_LOCAL)
        L.ref_paged_attention_v1.argtypes = [c_void_p] * 6 + [c_float] + [c_int32] * 7
        L.ref_reshape_and_cache.argtypes = [c_void_p] * 5 + [c_int32] * 4
        L.ref_copy_blocks.argtypes = [c_void_p] * 3 + [c_int32] * 4
        L.ref_swap_blocks.argtypes = [c_void_p] * 3 + [c_int32] * 2
        L.ref_compact_kv_cache.argtypes = [c_void_p] * 4 + [c_int32] * 4
        L.ref_memset_blocks.argtypes = [c_void_p] * 2 + [c_int32] * 2
        self.lib = L


class RefApi:
    """CacheFlow's cacheflow::cuda::launch_* call shape, compiled against its
    unchanged headers and linked to libcacheflow_b200.so (ref_api_driver.cpp):
    the reference-facing C++ entry points of the product, run on the GPU."""

    def __init__(self):
        if not REF_API_LIB.exists():
            raise FileNotFoundError(f"{REF_API_LIB} not built (make -C oracle ref)")
        L = ctypes.CDLL(str(REF_API_LIB), mode=os.RTLD_LOCAL)
        L.api_paged_attention_v1.argtypes = [c_void_p] * 6 + [c_float] + [c_int32] * 7 + [c_void_p]
        L.api_paged_attention_v2.argtypes = ([c_void_p] * 6 + [c_float] + [c_int32] * 7 + [c_void_p] * 3
                                             + [c_int32, c_void_p])
        L.api_reshape_and_cache.argtypes = [c_void_p] * 5 + [c_int32] * 4 + [c_void_p]
        L.api_copy_blocks.argtypes = [c_void_p] * 3 + [c_int32] * 4 + [c_void_p]
        L.api_swap_blocks.argtypes = [c_void_p] * 3 + [c_int32] * 2 + [c_void_p]
        L.api_compact_kv_cache.argtypes = [c_void_p] * 4 + [c_int32] * 4 + [c_void_p]
        L.api_memset_blocks.argtypes = [c_void_p] * 2 + [c_int32] * 2 + [c_void_p]
        L.api_async_memcpy_d2d.argtypes = [c_void_p, c_void_p, ctypes.c_size_t, c_void_p]
        L.api_synchronize_device.restype = None
        self.lib = L


class RefEngine:
    """CacheFlow's Scheduler / BatchManager / BlockManager (reference sources)
    over the C++ decode step of include/cacheflow_b200_engine.hpp
    (ref_engine_driver.cpp)."""

    COUNTS = ("rows", "swaps_out", "swaps_in", "copies", "seqs", "decode_rows", "chunks", "fused")

    def __init__(self, num_heads, num_kv_heads, head_dim, dtype_code, num_gpu_blocks, num_cpu_blocks, max_num_seqs,
                 max_batched_tokens, max_rows, max_blocks_per_seq, gpu_k, gpu_v, cpu_k, cpu_v):
        if not REF_ENGINE_LIB.exists():
            raise FileNotFoundError(f"{REF_ENGINE_LIB} not built (make -C oracle ref)")
        L = ctypes.CDLL(str(REF_ENGINE_LIB), mode=os.RTLD_LOCAL)
        L.eng_create.restype = c_void_p
        L.eng_create.argtypes = [c_int32] * 4 + [c_int64] * 2 + [c_int32] * 4 + [c_void_p] * 4 + [POINTER(c_int32)]
        L.eng_destroy.argtypes = [c_void_p]
        L.eng_add_request.argtypes = [c_void_p, ctypes.c_uint64, c_int32, c_int32]
        L.eng_has_pending.restype = c_int32
        L.eng_has_pending.argtypes = [c_void_p]
        L.eng_schedule.restype = c_int32
        L.eng_schedule.argtypes = [c_void_p, c_void_p, c_void_p]
        L.eng_rows.restype = c_int32
        L.eng_rows.argtypes = [c_void_p, c_void_p, c_void_p, c_void_p, c_int32]
        L.eng_block_ops.argtypes = [c_void_p, c_void_p, c_void_p, c_void_p]
        L.eng_attend.restype = c_int32
        L.eng_attend.argtypes = [c_void_p] * 6
        L.eng_finish_step.argtypes = [c_void_p, c_void_p, c_int32]
        self.lib = L
        st = c_int32(-1)
        self.h = L.eng_create(num_heads, num_kv_heads, head_dim, dtype_code, num_gpu_blocks, num_cpu_blocks,
                              max_num_seqs, max_batched_tokens, max_rows, max_blocks_per_seq, gpu_k, gpu_v, cpu_k,
                              cpu_v, ctypes.byref(st))
        if not self.h:
            raise RuntimeError(f"eng_create failed: status {st.value}")
        self.max_blocks = max_blocks_per_seq

    def add_request(self, rid: int, prompt_len: int, max_tokens: int) -> None:
        self.lib.eng_add_request(self.h, rid, prompt_len, max_tokens)

    def has_pending(self) -> bool:
        return bool(self.lib.eng_has_pending(self.h))

    def schedule(self, stream) -> dict:
        c = np.zeros(8, np.int32)
        st = self.lib.eng_schedule(self.h, stream, _p(c))
        if st != 0:
            raise RuntimeError(f"eng_schedule: status {st}")
        return dict(zip(self.COUNTS, (int(x) for x in c)))

    def rows(self, n: int):
        ids = np.zeros(max(n, 1), np.uint64)
        pos = np.zeros(max(n, 1), np.int32)
        tab = np.full((max(n, 1), self.max_blocks), -1, np.int32)
        if self.lib.eng_rows(self.h, _p(ids), _p(pos), _p(tab), self.max_blocks) != 0:
            raise RuntimeError("eng_rows failed")
        return ids[:n], pos[:n], tab[:n]

    def block_ops(self, counts: dict):
        out = np.zeros((max(counts["swaps_out"], 1), 2), np.int64)
        inn = np.zeros((max(counts["swaps_in"], 1), 2), np.int64)
        cp = np.zeros((max(counts["copies"], 1), 2), np.int64)
        self.lib.eng_block_ops(self.h, _p(out), _p(inn), _p(cp))
        return out[: counts["swaps_out"]], inn[: counts["swaps_in"]], cp[: counts["copies"]]

    def attend(self, q, out, k_new, v_new, stream) -> int:
        return self.lib.eng_attend(self.h, q, out, k_new, v_new, stream)

    def finish_step(self, tokens: np.ndarray) -> None:
        t = np.ascontiguousarray(tokens, np.int32)
        self.lib.eng_finish_step(self.h, _p(t) if t.size else None, int(t.size))

    def close(self) -> None:
        if self.h:
            self.lib.eng_destroy(self.h)
            self.h = None


class RefCpu:
    """CacheFlow's own CPU decode step (batch_decode.cpp:190-240), fp32 only."""

    def __init__(self, num_heads, num_kv_heads, head_dim, num_blocks, num_threads):
        if not REF_CPU_LIB.exists():
            raise FileNotFoundError(f"{REF_CPU_LIB} not built (make -C oracle ref)")
        L = ctypes.CDLL(str(REF_CPU_LIB), mode=os.RTLD_LOCAL)
        L.refcpu_create.restype = c_void_p
        L.refcpu_create.argtypes = [c_int32, c_int32, c_int32, c_int64, c_int32]
        L.refcpu_key_cache.restype = c_void_p
        L.refcpu_key_cache.argtypes = [c_void_p]
        L.refcpu_value_cache.restype = c_void_p
        L.refcpu_value_cache.argtypes = [c_void_p]
        L.refcpu_set_batch.argtypes = [c_void_p, c_int32, c_void_p, c_void_p, c_int32]
        L.refcpu_step.restype = c_double
        L.refcpu_step.argtypes = [c_void_p]
        L.refcpu_destroy.argtypes = [c_void_p]
        L.refcpu_prepare_inputs.restype = c_int32
        L.refcpu_prepare_inputs.argtypes = [c_void_p, c_int32, c_void_p, c_void_p, c_void_p, c_int32, c_void_p,
                                            c_void_p, c_void_p, c_void_p]
        self.lib = L
        self.shape = (num_blocks, num_kv_heads, 16, head_dim)
        self.h = L.refcpu_create(num_heads, num_kv_heads, head_dim, num_blocks, num_threads)
        self.num_threads = num_threads

    def caches(self) -> tuple[np.ndarray, np.ndarray]:
        n = int(np.prod(self.shape))
        k = np.ctypeslib.as_array(ctypes.cast(self.lib.refcpu_key_cache(self.h), POINTER(c_float)), (n,))
        v = np.ctypeslib.as_array(ctypes.cast(self.lib.refcpu_value_cache(self.h), POINTER(c_float)), (n,))
        return k.reshape(self.shape), v.reshape(self.shape)

    def set_batch(self, context_lens: np.ndarray, block_tables: np.ndarray) -> None:
        self._cl = np.ascontiguousarray(context_lens, dtype=np.int32)
        self._bt = np.ascontiguousarray(block_tables, dtype=np.int32)
        self.lib.refcpu_set_batch(self.h, self._cl.shape[0], _p(self._cl), _p(self._bt), self._bt.shape[1])

    def step(self) -> float:
        return float(self.lib.refcpu_step(self.h))

    def prepare_inputs(self, positions, block_offsets, block_ids):
        """The reference's prepare_kv_cache_inputs on CSR rows: (tables, context_lens, slots)."""
        pos = np.ascontiguousarray(positions, dtype=np.int32)
        off = np.ascontiguousarray(block_offsets, dtype=np.int64)
        ids = np.ascontiguousarray(block_ids, dtype=np.int32)
        if ids.size == 0:
            ids = np.zeros(1, np.int32)
        S = pos.shape[0]
        cap = int(np.diff(off).max()) if S else 0
        tables = np.zeros((S, max(cap, 1)), np.int32)
        ctx = np.zeros(S, np.int32)
        slots = np.zeros(S, np.int32)
        mb = c_int32(0)
        rc = self.lib.refcpu_prepare_inputs(self.h, S, _p(pos), _p(off), _p(ids), tables.shape[1], _p(tables),
                                            ctypes.byref(mb), _p(ctx), _p(slots))
        assert rc == 0
        return tables.reshape(-1)[: S * mb.value].reshape(S, mb.value), ctx, slots

    def close(self) -> None:
        if self.h:
            self.lib.refcpu_destroy(self.h)
            self.h = None
