"""The C-ABI library loads and exports every symbol include/fastb200.h declares; host-side
argument validation rejects bad calls before touching the GPU. CPU only: no compute calls."""

import ctypes
import os
import re

import pytest

import conftest

HEADER = os.path.join(conftest.ROOT, "include", "fastb200.h")


def declared():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(fb_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_entry_points():
    names = declared()
    for name in ("fb_decode_attention", "fb_decode_attention_combine", "fb_qk_norm_rope_append",
                 "fb_add_rmsnorm", "fb_rmsnorm", "fb_embed_rmsnorm", "fb_swiglu", "fb_linear", "fb_argmax"):
        assert name in names


def test_library_exports_every_declared_symbol():
    from kernels import _native
    lib = ctypes.CDLL(_native.LIBRARY_PATH)
    missing = [name for name in declared() if not hasattr(lib, name)]
    assert not missing, missing
    # the Python binding types every declared entry point
    assert sorted(_native.exported_names()) == declared()
    assert _native.lib.fb_version() >= 1


def test_host_validation_without_gpu():
    from kernels._native import lib
    null = None
    # null pointers -> FB_ERR_ARG, nothing launched
    assert lib.fb_decode_attention(null, null, null, null, 0, null, null, 0, 1, 16, 8, 128, 2048, 0.1, 148, null) == -1
    assert lib.fb_qk_norm_rope_append(null, 1, null, null, 1e-6, 1e-6, null, null, null, null, null, null, null,
                                      1, 1, 32, 8, 128, 9, 0, 0, null) == -1
    assert lib.fb_rmsnorm(null, 1024, null, null, 1, 1024, 1e-6, null) == -1
    assert lib.fb_argmax(null, 1, 100, null, null, null, 0, null) == -1
    p = ctypes.c_void_p(16)  # never dereferenced: shape checks fail first
    # unsupported shapes -> FB_ERR_SHAPE
    assert lib.fb_linear(p, p, p, 65, 128, 128, 0, 1, null) == -2     # > 64 rows
    assert lib.fb_linear(p, p, p, 4, 128, 100, 0, 1, null) == -2      # K not a multiple of 8
    assert lib.fb_linear(p, p, p, 4, 128, 128, 7, 1, null) == -1      # unknown epilogue
    assert lib.fb_linear(p, p, p, 4, 128, 128, 0, 3, null) == -2      # more splits than K chunks
    assert lib.fb_linear(p, p, p, 4, 128, 4096, 0, 9, null) == -2     # finished tile: a cluster of <= 8 splits
    assert lib.fb_linear_finished_splits(16, 3072, 4096) <= 8
    assert lib.fb_linear_finished_splits(64, 151936, 4096) <= 8
    # cluster-shape override: 2 to 16 CTAs, ring depth 2-4; (0, 0) restores automatic
    assert lib.fb_decode_attention_cluster_shape(1, 2) == -1
    assert lib.fb_decode_attention_cluster_shape(8, 5) == -1
    assert lib.fb_decode_attention_cluster_shape(17, 2) == -1
    assert lib.fb_decode_attention_cluster_shape(9, 4) == 0
    assert lib.fb_decode_attention_cluster_shape(0, 0) == 0
    assert lib.fb_swiglu(p, 1, p, 4, 12, null) == -2                     # width % 8
    assert lib.fb_add_rmsnorm(p, 1, p, p, p, p, 4, 70000, 1e-6, null) == -2  # row too wide (> 65536)
    assert lib.fb_decode_attention(p, p, p, p, 0, p, p, 1 << 20, 1, 16, 8, 96, 2048, 0.1, 148, null) == -2  # D=96
    assert lib.fb_decode_attention(p, p, p, p, 0, p, p, 1 << 20, 1, 72, 8, 128, 2048, 0.1, 148, null) == -2  # G=9
    # prefill attention: head_dim 96 and capacity < tokens are unsupported; null -> ARG
    assert lib.fb_prefill_attention(null, p, p, p, 1, 16, 8, 2, 128, 16, 0.1, null) == -1
    assert lib.fb_prefill_attention(p, p, p, p, 1, 16, 8, 2, 96, 16, 0.1, null) == -2
    assert lib.fb_prefill_attention(p, p, p, p, 1, 16, 8, 2, 128, 8, 0.1, null) == -2
    # speculation bookkeeping: blocks wider than 64 tokens, drafts outside [1, T-1]
    assert lib.fb_spec_propose(p, 64, p, p, 8, 4, p, p, p, p, 2, 65, 1, 1, 1, 1, 8, null) == -2
    assert lib.fb_spec_propose(p, 64, p, p, 8, 4, p, p, p, p, 2, 8, 0, 1, 1, 1, 8, null) == -1
    assert lib.fb_spec_propose(p, 64, p, p, 8, 4, p, p, p, p, 2, 8, 1, 1, 1, 8, 8, null) == -1
    assert lib.fb_spec_settle(p, p, null, p, p, p, 64, p, p, p, p, p, 2, 65, null) == -2
    assert lib.fb_spec_relocate(p, 4, 2, 2, 64, 60, p, p, null) == -2
    # tensor-parallel all-reduce: widths that do not split into even slices, unaligned peer
    # regions, bad ranks
    peers = (ctypes.c_void_p * 2)(16, 32)
    assert lib.fb_reduce_scatter_push(p, 2, 4, 6, 2, 0, 0, peers, p, null) == -2   # 6 % (2 * 2)
    assert lib.fb_reduce_scatter_push(p, 2, 4, 8, 2, 2, 0, peers, p, null) == -1   # rank >= world
    odd = (ctypes.c_void_p * 2)(16, 40)
    assert lib.fb_reduce_scatter_push(p, 2, 4, 8, 2, 0, 0, odd, p, null) == -1     # not 16-byte aligned
    assert lib.fb_allreduce_add_rmsnorm(p, p, p, peers, peers, 0, 9, 0, p, p, p, p, p, 4, 4096, 1e-6, null) == -1
    assert lib.fb_allreduce_add_rmsnorm(p, p, p, peers, peers, 0, 2, 0, p, p, p, p, p, 4, 4100, 1e-6, null) == -2
    assert lib.fb_allreduce_add_rmsnorm(null, p, p, peers, peers, 0, 2, 0, p, p, p, p, p, 4, 4096, 1e-6, null) == -1
    # push form: argument checks only (no launch)
    assert lib.fb_allreduce_push(p, 2, 4, 7, 2, 0, 0, peers, p, null) == -2       # odd width
    assert lib.fb_allreduce_push(p, 2, 4, 8, 2, 2, 0, peers, p, null) == -1       # rank >= world
    assert lib.fb_allreduce_push(p, 2, 4, 8, 2, 0, 0, odd, p, null) == -1         # not 16-byte aligned
    assert lib.fb_allreduce_sum_add_rmsnorm(p, 0, 9, p, p, p, p, p, 4, 4096, 1e-6, null) == -1  # world > 8
    assert lib.fb_allreduce_sum_add_rmsnorm(null, 0, 2, p, p, p, p, p, 4, 4096, 1e-6, null) == -1
    assert lib.fb_linear_argmax(p, p, 4, 128, 128, -1, p, null) == -1
    # workspace too small -> FB_ERR_WORKSPACE
    need = lib.fb_decode_attention_workspace(1, 16, 8, 128, 148)
    assert need > 0
    assert lib.fb_decode_attention(p, p, p, p, 0, p, p, need - 1, 1, 16, 8, 128, 2048, 0.1, 148, null) == -5


def test_workspace_sizes():
    from kernels._native import lib
    # (ctas + B*Hkv) slots of G*D fp32 partials plus G (max, sum) stats
    need = lib.fb_decode_attention_workspace(4, 32, 8, 128, 148)
    slots = 148 + 4 * 8
    assert need >= slots * 4 * 128 * 4 + slots * 4 * 8
    assert lib.fb_argmax_workspace(16, 151936) >= 16 * 19 * 8


def test_python_wrappers_refuse_cpu_tensors():
    import torch
    from kernels.rmsnorm import rms_norm
    with pytest.raises(ValueError):
        rms_norm(torch.zeros(2, 64, dtype=torch.bfloat16), torch.ones(64, dtype=torch.bfloat16), 1e-6)
