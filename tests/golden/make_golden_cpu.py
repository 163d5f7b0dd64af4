"""Records golden vectors from CacheFlow's OWN host code (oracle/_ref/
libcf_ref_cpu.so: batch_decode.cpp and memory_pool.cpp compiled from the
reference sources by oracle/Makefile, plus oracle/ref_cpu_driver.cpp).
Needs no GPU:

    make -C oracle ref && python tests/golden/make_golden_cpu.py tests/golden

build_decode_inputs.npz: seeded decode batches run through the reference's
BatchDecodeEngine::prepare_kv_cache_inputs (batch_decode.cpp:92-131); holds
the CSR inputs (positions, block_offsets, block_ids), its block tables,
context lengths and slot mapping, and `slot_set` -- the rows whose slot the
reference writes (position / 16 < number of blocks, :110); the others hold
whatever its uninitialised array held and are stored as -1.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))


def main(out_dir: str) -> None:
    from oracle import oracle

    out = Path(out_dir)
    out.mkdir(parents=True, exist_ok=True)
    rng = np.random.default_rng(20261202)
    ref = oracle.RefCpu(num_heads=1, num_kv_heads=1, head_dim=16, num_blocks=16, num_threads=1)
    try:
        S = 96
        nblk = rng.integers(0, 40, S)
        nblk[:6] = [0, 1, 1, 2, 39, 7]
        pos = np.array([min(int(rng.integers(0, max(n, 1) * 16)), max(n * 16 - 1, 0)) for n in nblk], np.int32)
        # edge positions: first / last slot of a block, and rows whose
        # position is past their blocks (the reference leaves those slots unset)
        pos[:6] = [0, 0, 15, 16, 39 * 16 - 1, 7 * 16 + 3]
        pos[6] = nblk[6] * 16 + 20
        off = np.zeros(S + 1, np.int64)
        off[1:] = np.cumsum(nblk)
        ids = rng.permutation(200000)[: int(off[-1])].astype(np.int32)
        tables, ctx, slots = ref.prepare_inputs(pos, off, ids)
        slot_set = (pos // 16) < nblk
        slots = np.where(slot_set, slots, -1).astype(np.int32)
        np.savez_compressed(out / "build_decode_inputs.npz", op="build_decode_inputs", positions=pos,
                            block_offsets=off, block_ids=ids, block_tables=tables, context_lens=ctx,
                            slot_mapping=slots, slot_set=slot_set)
    finally:
        ref.close()


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else str(Path(__file__).resolve().parent))
