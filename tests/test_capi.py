"""CPU-side checks of the drop-in boundary: the library loads, exports exactly
what include/*.h declares, rejects bad arguments before touching the GPU, and
its host-only planners behave.  No compute calls (there is no GPU here)."""

import ctypes
import os
import re
import shutil
import subprocess
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]


def _declared_c_functions():
    text = (ROOT / "include" / "cacheflow_b200.h").read_text()
    return re.findall(r"CF_API\s+[\w\s\*]+?\b(cf_\w+)\s*\(", text)


def _exports(lib_path):
    out = subprocess.run(["nm", "-D", "--defined-only", str(lib_path)], capture_output=True, text=True,
                         check=True).stdout
    names = {line.split()[-1] for line in out.splitlines() if " T " in line}
    demangled = subprocess.run(["c++filt"], input="\n".join(sorted(names)), capture_output=True, text=True,
                               check=True).stdout.splitlines()
    return names, set(demangled)


def test_library_exports_every_declared_c_function(cflib):
    from cacheflow_b200 import _lib

    declared = set(_declared_c_functions())
    assert declared == set(_lib.SIGNATURES), "ctypes binding and header disagree"
    names, _ = _exports(_lib.LIB_PATH)
    assert declared <= names
    for n in declared:
        assert getattr(cflib, n) is not None


def test_library_exports_reference_cpp_entry_points(cflib):
    from cacheflow_b200 import _lib

    _, demangled = _exports(_lib.LIB_PATH)
    for sym in _lib.COMPAT_SYMBOLS:
        assert sym in demangled, sym
    # nothing but the ABI is exported
    extra = {d for d in demangled if not (d.startswith("cf_") or d.startswith("cacheflow::cuda::"))}
    assert not extra, extra


def test_compat_header_declares_reference_signatures():
    """Every C++ entry point of the compat header is exported (same mangling as
    CacheFlow's own declarations, checked below when its sources are present)."""
    text = (ROOT / "include" / "cacheflow_b200_compat.hpp").read_text()
    for fn in ["launch_paged_attention_v1", "launch_paged_attention_v2", "launch_reshape_and_cache",
               "launch_copy_blocks", "launch_swap_blocks", "launch_compact_kv_cache", "launch_memset_blocks",
               "get_gpu_free_memory", "async_memcpy_h2d", "synchronize_stream"]:
        assert re.search(rf"CF_COMPAT_API\s+\w+\s+{fn}\(", text), fn


def _reference_dir():
    from oracle import oracle

    return oracle.reference_dir()


REF = _reference_dir()


@pytest.mark.skipif(REF is None or shutil.which("g++") is None, reason="CacheFlow sources not present")
def test_reference_host_code_links_against_library(cflib, tmp_path):
    """CacheFlow's own decode engine, compiled with CUDA enabled against its own
    unchanged headers, links against libcacheflow_b200.so with no undefined
    cacheflow::cuda symbol: the library is a drop-in for src/cacheflow/cuda/*.cu."""
    from cacheflow_b200 import _lib

    src = REF / "src"
    out = tmp_path / "libengine.so"
    cmd = ["g++", "-std=c++17", "-O1", "-fPIC", "-shared", "-DCACHEFLOW_USE_CUDA=1", f"-I{src}",
           "-I/usr/local/cuda/include", str(src / "cacheflow/decode/batch_decode.cpp"),
           str(src / "cacheflow/kv_cache/memory_pool.cpp"), "-o", str(out),
           f"-L{_lib.LIB_PATH.parent}", "-lcacheflow_b200", "-Wl,--no-undefined",
           "-L/usr/local/cuda/lib64", "-lcudart"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-3000:]
    und = subprocess.run(["nm", "-D", "-C", "--undefined-only", str(out)], capture_output=True, text=True).stdout
    used = [l for l in und.splitlines() if "cacheflow::cuda::" in l]
    assert any("launch_paged_attention_v1" in l for l in used)
    assert any("launch_paged_attention_v2" in l for l in used)


def test_invalid_arguments_rejected_without_gpu(cflib):
    from cacheflow_b200 import _lib

    assert cflib.cf_abi_version() == 1
    assert cflib.cf_paged_attention_v1(None, None, 0, None) == _lib.CF_ERR_INVALID_ARGUMENT
    p = _lib.AttentionParams()
    p.num_seqs, p.num_heads, p.num_kv_heads, p.head_dim, p.block_size = 1, 6, 4, 128, 16
    p.dtype = _lib.CF_BF16
    assert cflib.cf_paged_attention_v1(ctypes.byref(p), None, 0, None) == _lib.CF_ERR_INVALID_ARGUMENT
    p.num_kv_heads, p.head_dim = 2, 96
    assert cflib.cf_paged_attention_v1(ctypes.byref(p), None, 0, None) == _lib.CF_ERR_UNSUPPORTED
    p.head_dim, p.block_size = 128, 32
    assert cflib.cf_paged_attention_v1(ctypes.byref(p), None, 0, None) == _lib.CF_ERR_UNSUPPORTED
    p.block_size, p.max_blocks_per_seq, p.max_context_len = 16, 2, 33  # 33 tokens > 2 blocks
    assert cflib.cf_paged_attention_v1(ctypes.byref(p), None, 0, None) == _lib.CF_ERR_INVALID_ARGUMENT
    p.max_context_len, p.num_seqs = 10, 0  # empty batch is a no-op
    assert cflib.cf_paged_attention_v1(ctypes.byref(p), None, 0, None) == _lib.CF_OK
    p.num_seqs, p.max_context_len = 1, 600
    p.query = p.key_cache = p.value_cache = p.output = p.block_tables = p.context_lens = 1 << 20
    p.max_blocks_per_seq = 64
    es = ctypes.c_void_p(1 << 20)
    assert cflib.cf_paged_attention_v2(ctypes.byref(p), es, es, es, 1, None) == _lib.CF_ERR_WORKSPACE
    assert cflib.cf_reshape_and_cache(None, None, None, None, None, 0, 8, 128, 16, 10, 2, None) == _lib.CF_OK
    assert cflib.cf_reshape_and_cache(None, None, None, None, None, 4, 8, 128, 16, 10, 2, None) == \
        _lib.CF_ERR_INVALID_ARGUMENT
    assert cflib.cf_copy_blocks(None, None, None, -1, 8, 128, 16, 10, 2, None) == _lib.CF_ERR_INVALID_ARGUMENT
    assert cflib.cf_swap_blocks(None, None, None, 3, 4096, None) == _lib.CF_ERR_INVALID_ARGUMENT
    assert cflib.cf_compact_kv_cache(None, None, None, None, 0, 8, 128, 16, 10, 7, None) == \
        _lib.CF_ERR_INVALID_ARGUMENT
    assert cflib.cf_memset_blocks(None, None, 0, 4096, 10, None) == _lib.CF_OK
    assert cflib.cf_status_string(_lib.CF_ERR_PLAN) == b"block-move plan would race"
    # fused append: the new rows are required and 16-byte aligned
    assert cflib.cf_paged_attention_append_v1(ctypes.byref(p), None, None, None, None, 0, None) == \
        _lib.CF_ERR_INVALID_ARGUMENT
    assert cflib.cf_paged_attention_append_v2(ctypes.byref(p), (1 << 20) + 8, 1 << 20, None, es, es, es, 1,
                                              None) == _lib.CF_ERR_INVALID_ARGUMENT
    assert cflib.cf_paged_attention_append_v2(ctypes.byref(p), 1 << 20, 1 << 20, None, es, es, es, 1, None) == \
        _lib.CF_ERR_INVALID_ARGUMENT  # num_blocks 0: the appended ids could not be range-checked
    p.num_blocks = 64
    assert cflib.cf_paged_attention_append_v2(ctypes.byref(p), 1 << 20, 1 << 20, None, es, es, es, 1, None) == \
        _lib.CF_ERR_WORKSPACE
    # fused fp8 append: scales finite and > 0, rows present, then the v2 scratch rules
    assert cflib.cf_paged_attention_fp8_append_v2(ctypes.byref(p), 0.0, 1.0, 1 << 20, 1 << 20, None, es, es, es, 1,
                                                  None) == _lib.CF_ERR_INVALID_ARGUMENT
    assert cflib.cf_paged_attention_fp8_append_v1(ctypes.byref(p), 1.0, 1.0, None, 1 << 20, None, None, 0,
                                                  None) == _lib.CF_ERR_INVALID_ARGUMENT
    assert cflib.cf_paged_attention_fp8_append_v2(ctypes.byref(p), 0.5, 1.0, 1 << 20, 1 << 20, None, es, es, es, 1,
                                                  None) == _lib.CF_ERR_WORKSPACE
    # scheduler block ops: ids are range-checked on the host before anything runs
    pairs = (ctypes.c_int64 * 2)(0, 5)
    assert cflib.cf_execute_block_ops(None, None, None, None, 4096, 4, 4, None, 0, None, 0, None, 0, None) == _lib.CF_OK
    assert cflib.cf_execute_block_ops(1 << 20, 1 << 20, 1 << 21, 1 << 21, 4096, 8, 4, pairs, 1, None, 0, None, 0,
                                      None) == _lib.CF_ERR_INVALID_ARGUMENT  # cpu id 5 >= 4
    # decode-input builder
    assert cflib.cf_build_decode_inputs(None, None, None, 0, 4, 16, None, None, None, None) == _lib.CF_OK
    assert cflib.cf_build_decode_inputs(None, None, None, 3, 4, 16, None, None, None, None) == \
        _lib.CF_ERR_INVALID_ARGUMENT
    assert cflib.cf_build_decode_inputs(None, None, None, 3, 0, 16, None, None, None, None) == \
        _lib.CF_ERR_INVALID_ARGUMENT


def test_compaction_planner_packs_without_overlap(cflib):
    from cacheflow_b200 import _lib, ops

    rng = np.random.default_rng(0)
    for n, frac in [(1, 1.0), (10, 0.0), (1000, 0.5), (4096, 0.9), (777, 0.1)]:
        used = rng.random(n) < frac
        src, dst = ops.compaction_plan(used)
        live = int(used.sum())
        assert ops.check_compaction_plan(src, dst, n) == _lib.CF_OK
        assert np.all(src >= live) and np.all(dst < live)
        after = used.copy()
        after[src] = False
        after[dst] = True
        assert after[:live].all() and not after[live:].any()


def test_plan_checker_rejects_races(cflib):
    from cacheflow_b200 import _lib, ops

    assert ops.check_compaction_plan(np.array([5, 6]), np.array([1, 1]), 10) == _lib.CF_ERR_PLAN  # dup dst
    assert ops.check_compaction_plan(np.array([5, 1]), np.array([1, 2]), 10) == _lib.CF_ERR_PLAN  # chain
    assert ops.check_compaction_plan(np.array([5]), np.array([10]), 10) == _lib.CF_ERR_INVALID_ARGUMENT
    assert ops.check_compaction_plan(np.array([4, 4]), np.array([4, 7]), 10) == _lib.CF_OK  # self move skipped


def test_v1_workspace_size_needs_shapes_only(cflib):
    """The size query is answered from host-side fields; no operand pointers."""
    from cacheflow_b200 import _lib

    p = _lib.AttentionParams()
    p.num_seqs, p.num_heads, p.num_kv_heads, p.head_dim, p.block_size = 64, 32, 32, 128, 16
    p.max_context_len, p.max_blocks_per_seq, p.dtype = 4096, 256, _lib.CF_F16
    n = cflib.cf_paged_attention_v1_workspace_size(ctypes.byref(p))
    parts = 4096 // 2048
    rows = 64 * 32 * parts
    assert n >= rows * (128 + 2) * 4
    p.max_context_len = 1000  # fits one partition: never splits
    assert cflib.cf_paged_attention_v1_workspace_size(ctypes.byref(p)) == 0


def _split_bytes(rows, D):
    r = lambda b: (b + 255) // 256 * 256
    return 2 * r(rows * 4) + r(rows * D * 4)


def test_v1_split_policy(cflib):
    """Partitions of 2048 tokens, 4096 past 8192 tokens (2048 for an fp8 cache,
    8192 with 4096 or more row x KV head pairs), halved (not below 512) while
    the grid would hold fewer than ~4 CTAs per SM of 148; the workspace covers
    every shorter context and both cache types."""
    import os

    from cacheflow_b200 import _lib

    if os.environ.get("CF_V1_SPLIT_TOKENS"):
        pytest.skip("CF_V1_SPLIT_TOKENS overrides the policy")
    p = _lib.AttentionParams()
    p.num_heads, p.head_dim, p.block_size, p.dtype = 32, 128, 16, _lib.CF_BF16
    size = lambda: cflib.cf_paged_attention_v1_workspace_size(ctypes.byref(p))  # noqa: E731
    # 16 rows x 8 kv heads up to 124,872 tokens: 4096-token partitions (31),
    # 2048 for an fp8 cache (61), which sets the size
    p.num_seqs, p.num_kv_heads, p.max_context_len, p.max_blocks_per_seq = 16, 8, 124872, 7805
    assert size() == _split_bytes(16 * 32 * 61, 128)
    # 64 rows x 32 kv heads up to 4096 tokens: 2048-token partitions (2)
    p.num_seqs, p.num_kv_heads, p.max_context_len, p.max_blocks_per_seq = 64, 32, 4096, 256
    assert size() == _split_bytes(64 * 32 * 2, 128)
    # 2 rows x 8 kv heads up to 20,000 tokens: 4096 gives 80 CTAs ... 512 640
    p.num_seqs, p.num_kv_heads, p.max_context_len, p.max_blocks_per_seq = 2, 8, 20000, 1250
    assert size() == _split_bytes(2 * 32 * 40, 128)
    # 1024 rows x 8 kv heads (8192 pairs) up to 32,659 tokens: 8192-token partitions (4)
    p.num_heads = 64
    p.num_seqs, p.num_kv_heads, p.max_context_len, p.max_blocks_per_seq = 1024, 8, 32659, 2042
    assert size() == _split_bytes(1024 * 64 * 4, 128)
    # 16 rows x 8 kv heads up to 10,000 tokens: the call itself needs 5
    # partitions (4096 -> 2048), one of 8192 tokens 8 (2048 -> 1024): the
    # workspace is sized for 8
    p.num_heads = 32
    p.num_seqs, p.num_kv_heads, p.max_context_len, p.max_blocks_per_seq = 16, 8, 10000, 625
    assert size() == _split_bytes(16 * 32 * 8, 128)


def test_engine_rejects_unknown_kernel_choice_before_touching_a_gpu():
    import torch

    from cacheflow_b200.engine import DecodeEngine

    with pytest.raises(ValueError):
        DecodeEngine(torch.empty((4, 2, 16, 64)), torch.empty((4, 2, 16, 64)), 2, 1, 1, kernel="v3")


@pytest.mark.skipif(shutil.which("g++") is None, reason="g++ not present")
def test_engine_header_compiles_against_cacheflow_shaped_types(tmp_path):
    """include/cacheflow_b200_engine.hpp needs only the C ABI header and the
    CUDA runtime: it compiles warning-free against types with the fields of
    CacheFlow's DecodeBatch and SchedulerOutput (batch_manager.h:13-36,
    scheduler.h:16-30) without CacheFlow's headers."""
    src = tmp_path / "use_engine.cpp"
    src.write_text(
        "#include \"cacheflow_b200_engine.hpp\"\n"
        "#include <cstdint>\n#include <vector>\n"
        "struct Entry { uint64_t seq_id; int32_t token; int32_t position; std::vector<int32_t> block_table;"
        " bool is_prefill; };\n"
        "struct Batch { std::vector<Entry> entries; size_t total_tokens = 0; };\n"
        "struct BlockOp { uint64_t seq_id; int32_t src; int32_t dst; };\n"
        "struct Output { std::vector<BlockOp> block_copies, block_swaps_in, block_swaps_out; };\n"
        "int run(void* k, void* v, void* q, void* o, cudaStream_t s) {\n"
        "  cacheflow_b200::StepShape sh; sh.num_heads = 32; sh.num_kv_heads = 8; sh.head_dim = 128;\n"
        "  sh.num_gpu_blocks = 1024; sh.max_rows = 256; sh.max_blocks_per_seq = 512;\n"
        "  cacheflow_b200::DecodeStep step(sh, k, v);\n"
        "  Batch b; b.entries.push_back({1, 7, 20, {3, 4}, false}); Output so;\n"
        "  if (step.execute_block_ops(so, s) != CF_OK) return 1;\n"
        "  if (step.stage(b, s) != CF_OK) return 2;\n"
        "  return step.attend(q, o, nullptr, nullptr, s);\n"
        "}\n")
    r = subprocess.run(["g++", "-std=c++17", "-Wall", "-Wextra", "-Werror", "-fsyntax-only", f"-I{ROOT / 'include'}",
                        "-I/usr/local/cuda/include", str(src)], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-3000:]
