"""Records golden vectors from CacheFlow's OWN CUDA kernels (oracle/_ref/
libcf_ref_cuda.so, compiled from the reference sources by oracle/Makefile).

Run on a CUDA machine from the repository root:

    python tests/golden/make_golden.py <out_dir>

Each .npz holds the seeded inputs of one operator call and the reference
kernel's outputs; tests/test_oracle.py checks that the CPU oracle reproduces
them (bit-exact for data movement, 1e-5 for fp32 attention).  Only inputs the
reference handles correctly are recorded: fp32 everywhere (its only type) and
attention contexts <= 128 tokens (its V1 shared array holds 128 scores).
"""

from __future__ import annotations

import math
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "tests"))


def main(out_dir: str) -> None:
    import torch

    from helpers import random_tables
    from oracle import oracle

    out = Path(out_dir)
    out.mkdir(parents=True, exist_ok=True)
    L = oracle.RefCuda().lib
    rng = np.random.default_rng(20261201)
    dev = torch.device("cuda:0")

    def d(a):
        return torch.from_numpy(np.ascontiguousarray(a)).to(dev)

    def f32(shape):
        return rng.standard_normal(shape, dtype=np.float32)

    # paged attention V1, two head shapes, contexts up to 128 tokens
    for D, H, Hkv in [(128, 4, 2), (64, 4, 4)]:
        ctx = np.array([1, 15, 16, 17, 64, 100, 128], np.int32)
        pool = int(((ctx + 15) // 16).sum()) + 4
        tables = random_tables(rng, ctx.tolist(), pool)
        q, k, v = f32((len(ctx), H, D)), f32((pool, Hkv, 16, D)), f32((pool, Hkv, 16, D))
        o = torch.zeros((len(ctx), H, D), device=dev)
        dq, dk, dv, bt, cl = d(q), d(k), d(v), d(tables), d(ctx)
        scale = np.float32(1.0 / math.sqrt(D))
        assert L.ref_paged_attention_v1(dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), o.data_ptr(), bt.data_ptr(),
                                        cl.data_ptr(), float(scale), len(ctx), H, Hkv, D, 16, int(ctx.max()),
                                        tables.shape[1]) == 0
        np.savez_compressed(out / f"paged_attention_v1_d{D}_h{H}_kv{Hkv}.npz", op="paged_attention_v1", q=q, k=k,
                            v=v, block_tables=tables, context_lens=ctx, scale=scale, out=o.cpu().numpy())

    pool, Hkv, D = 24, 2, 64
    kc, vc = f32((pool, Hkv, 16, D)), f32((pool, Hkv, 16, D))
    T = 40
    key, val = f32((T, Hkv, D)), f32((T, Hkv, D))
    slots = np.concatenate([[0, pool * 16 - 1], 1 + rng.permutation(pool * 16 - 2)[: T - 2]]).astype(np.int32)
    # every device tensor stays referenced until the kernel has finished
    a, b, dkey, dval, dslots = d(kc), d(vc), d(key), d(val), d(slots)
    assert L.ref_reshape_and_cache(dkey.data_ptr(), dval.data_ptr(), a.data_ptr(), b.data_ptr(),
                                   dslots.data_ptr(), T, Hkv, D, 16) == 0
    np.savez_compressed(out / "reshape_and_cache.npz", op="reshape_and_cache", key=key, value=val, k_cache=kc,
                        v_cache=vc, slot_mapping=slots, k_out=a.cpu().numpy(), v_out=b.cpu().numpy())

    ids = rng.permutation(pool)
    pairs = np.stack([ids[:6], ids[6:12]], 1).astype(np.int64)
    a, b, dpairs = d(kc), d(vc), d(pairs)
    assert L.ref_copy_blocks(a.data_ptr(), b.data_ptr(), dpairs.data_ptr(), len(pairs), Hkv, D, 16) == 0
    np.savez_compressed(out / "copy_blocks.npz", op="copy_blocks", k_cache=kc, v_cache=vc, block_mapping=pairs,
                        k_out=a.cpu().numpy(), v_out=b.cpu().numpy())

    dst = f32((10, Hkv, 16, D))
    sp = np.stack([ids[:5], np.array([9, 0, 4, 2, 7])], 1).astype(np.int64)
    a, b, dsp = d(kc), d(dst), d(sp)
    assert L.ref_swap_blocks(a.data_ptr(), b.data_ptr(), dsp.data_ptr(), len(sp), Hkv * 16 * D * 4) == 0
    np.savez_compressed(out / "swap_blocks.npz", op="swap_blocks", src=kc, dst=dst, block_mapping=sp,
                        dst_out=b.cpu().numpy())

    used = rng.random(pool) < 0.5
    live = int(used.sum())
    holes = [i for i in range(live) if not used[i]]
    movers = [i for i in range(live, pool) if used[i]]
    src, dstids = np.array(movers, np.int32), np.array(holes[: len(movers)], np.int32)
    a, b, dsrc, ddst = d(kc), d(vc), d(src), d(dstids)
    assert L.ref_compact_kv_cache(a.data_ptr(), b.data_ptr(), dsrc.data_ptr(), ddst.data_ptr(), len(src),
                                  Hkv, D, 16) == 0
    np.savez_compressed(out / "compact_kv_cache.npz", op="compact_kv_cache", k_cache=kc, v_cache=vc, src_ids=src,
                        dst_ids=dstids, k_out=a.cpu().numpy(), v_out=b.cpu().numpy())

    bids = np.array([0, 5, pool - 1], np.int32)
    a, dbids = d(kc), d(bids)
    assert L.ref_memset_blocks(a.data_ptr(), dbids.data_ptr(), len(bids), Hkv * 16 * D * 4) == 0
    np.savez_compressed(out / "memset_blocks.npz", op="memset_blocks", cache=kc, block_ids=bids,
                        out=a.cpu().numpy())
    print("golden vectors written to", out)


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "tests/golden")
