"""The C-ABI library: builds, loads without a GPU, exports every symbol the
header declares, and rejects bad arguments before touching the device."""
from __future__ import annotations

import ctypes
import os
import re

import pytest

from conftest import PKG, ROOT

HEADER = os.path.join(ROOT, "include", "moe_b200.h")


@pytest.fixture(scope="module")
def lib():
    import build as moe_build

    moe_build.build()
    import moe_host

    return moe_host.load_library()


def declared_functions() -> list[str]:
    text = open(HEADER).read()
    return sorted(set(re.findall(r"MOE_B200_API\s+[\w\s\*]+?\b(moe_b200_\w+)\s*\(", text)))


def test_header_declares_the_entry_points():
    names = declared_functions()
    for n in ("moe_b200_run", "moe_b200_route", "moe_b200_workspace_bytes", "moe_b200_read_status",
              "moe_b200_status_string", "moe_b200_get_workspace_layout", "moe_b200_set_stage_events",
              "moe_b200_abi_version", "moe_b200_ep_area_bytes", "moe_b200_ep_combine", "moe_b200_run_noalloc",
              "moe_b200_quantize_hidden", "moe_b200_run_bf16_hidden", "moe_b200_run_routing",
              "moe_b200_route_method"):
        assert n in names


def test_host_constants_match_the_header():
    import moe_host

    text = open(HEADER).read()

    def define(name):
        return int(re.search(rf"#define\s+{name}\s+(\d+)", text).group(1))

    assert moe_host.MAX_TOKENS == define("MOE_B200_MAX_TOKENS")
    assert moe_host.EP_COUNTER_BYTES == define("MOE_B200_EP_COUNTER_BYTES")
    assert moe_host.A2A_COUNTER_BYTES == define("MOE_B200_A2A_COUNTER_BYTES")


def test_library_exports_every_declared_symbol(lib):
    for name in declared_functions():
        assert hasattr(lib, name), f"{name} declared in moe_b200.h but not exported"


def test_library_is_sm100a_only():
    import build as moe_build

    assert moe_build.ARCH_FLAGS == ["-gencode", "arch=compute_100a,code=sm_100a"]
    assert os.path.exists(os.path.join(PKG, "libmoe_b200.so"))


def test_workspace_size_and_layout(lib):
    import moe_host

    assert moe_host.workspace_bytes(-1) == 0
    assert moe_host.workspace_bytes(moe_host.MAX_TOKENS + 1) == 0
    prev = 0
    for T in (0, 1, 16, 64, 65, 4096, 16384):
        n = moe_host.workspace_bytes(T)
        assert n > 0 and n % 256 == 0
        lay = moe_host.workspace_layout(T)
        assert lay.total_bytes == n
        assert lay.cap_rows == (8 * T + 15) // 16 * 16 + 32 * 16 + 128
        decode = T <= 64
        offs = [lay.counts, lay.seg_off, lay.chunk_counts, lay.topk_idx, lay.topk_w, lay.perm_tok, lay.perm_w,
                lay.perm_row, lay.tok_slot, lay.a_perm, lay.sa_perm, lay.c_hi, lay.c_lo, lay.c_scale, lay.y_acc]
        assert lay.status < lay.sched < lay.n_touched < lay.seg_off
        assert lay.a_perm - lay.tok_slot >= 4 * T and lay.tok_slot - lay.perm_row >= 4 * lay.cap_rows
        token_major = T >= moe_host.TOKEN_MAJOR_MIN_TOKENS
        if decode or token_major:
            offs += [lay.g1_acc]
        offs += [lay.slot_tok]   # appended after the others, so their offsets did not move
        if not decode:
            offs += [lay.hidden_q, lay.hidden_qs]
            assert lay.hidden_qs - lay.hidden_q >= T * 7168 and n - lay.hidden_qs >= 56 * 4 * T
            assert lay.hidden_q - lay.slot_tok >= 4 * T
        else:
            assert lay.hidden_q == 0 and lay.hidden_qs == 0
            assert n - lay.slot_tok >= 4 * T
        assert offs == sorted(offs) and all(o % 256 == 0 for o in offs)
        assert lay.c_lo - lay.c_hi >= lay.cap_rows * 2048
        if decode:
            assert lay.g1_acc - lay.y_acc >= T * 7168 * 4
            assert lay.slot_tok - lay.g1_acc >= lay.cap_rows * 4096 * 4
        elif token_major:
            # K-split GEMM1 sums of batches with few token tiles: 1,664 rows
            assert lay.g1_acc - lay.y_acc >= T * 7168 * 4
            assert lay.slot_tok - lay.g1_acc >= 1664 * 4096 * 4
        else:
            assert lay.g1_acc == 0
        if T > 65:  # plans without the decode scratch grow with T
            assert n >= prev
        prev = n


def test_status_strings(lib):
    import moe_host

    assert moe_host.status_string(0) == "ok"
    for code in range(1, 8):
        assert moe_host.status_string(code) not in ("ok", "unknown status")
    assert moe_host.status_string(99) == "unknown status"


def test_run_rejects_bad_arguments_without_a_device(lib):
    P = ctypes.c_void_p
    good = ctypes.create_string_buffer(4096 + 256)
    base = (ctypes.addressof(good) + 255) // 256 * 256
    p = P(base)
    args_null = [None, None, 0, None, None, None, None, None, None, 0, 2.5, 4, None, None, 0, None]
    assert lib.moe_b200_run(*args_null) == 1                       # null pointers
    full = [p, p, 0, p, p, p, p, p, p, 0, 2.5, 4, p, p, 1 << 40, None]
    full[11] = -1
    assert lib.moe_b200_run(*full) == 1                            # negative T
    full[11] = 4
    full[2] = 7
    assert lib.moe_b200_run(*full) == 1                            # bad bias dtype code
    full[2] = 0
    full[3] = P(base + 1)
    assert lib.moe_b200_run(*full) == 2                            # misaligned hidden_states
    full[3] = p
    full[13] = P(base + 16)
    assert lib.moe_b200_run(*full) == 2                            # misaligned workspace
    full[13] = p
    full[14] = 16
    assert lib.moe_b200_run(*full) == 3                            # workspace too small
    full[11] = 0
    assert lib.moe_b200_run(*full) == 0                            # T = 0 is a no-op
    assert lib.moe_b200_route(None, None, 0, 4, 2.5, None, None, None) == 1
    assert lib.moe_b200_route(p, p, 0, 0, 2.5, p, p, None) == 0
    assert lib.moe_b200_set_stage_events(None, 0) == 0
    assert lib.moe_b200_abi_version() == 9


def test_widened_entry_points_reject_bad_arguments_without_a_device(lib):
    """The routing-method, quantiser and bf16-hidden entry points check their
    arguments before any CUDA call."""
    P = ctypes.c_void_p
    buf = ctypes.create_string_buffer(4096 + 256)
    base = (ctypes.addressof(buf) + 255) // 256 * 256
    p = P(base)
    big = 1 << 40
    # unknown method, top_k outside 1..8, DeepSeek-V3 needs 8 picks, Llama4 one
    for method, top_k in [(6, 8), (-1, 8), (2, 4), (3, 2), (1, 0), (1, 9)]:
        assert lib.moe_b200_route_method(method, top_k, p, p, 0, 4, 1.0, p, p, None) == 1
        assert lib.moe_b200_run_routing(method, top_k, p, p, 0, p, p, p, p, p, p, 0, 1.0, 4, p, p, big, None) == 1
    assert lib.moe_b200_route_method(2, 8, p, None, 0, 4, 1.0, p, p, None) == 1    # DeepSeek-V3 needs its bias
    assert lib.moe_b200_route_method(1, 8, p, None, 0, 0, 1.0, p, p, None) == 0    # T = 0, bias optional
    assert lib.moe_b200_run_routing(1, 8, p, None, 0, p, p, p, p, p, p, 0, 1.0, 0, p, p, big, None) == 0
    assert lib.moe_b200_run_routing(3, 1, p, None, 0, P(base + 1), p, p, p, p, p, 0, 1.0, 4, p, p, big,
                                    None) == 2                                      # misaligned hidden_states
    assert lib.moe_b200_run_routing(5, 4, p, None, 0, p, p, p, p, p, p, 0, 1.0, 4, p, p, 16, None) == 3
    # the quantiser
    assert lib.moe_b200_quantize_hidden(None, 4, None, None, None) == 1
    assert lib.moe_b200_quantize_hidden(p, -1, p, p, None) == 1
    assert lib.moe_b200_quantize_hidden(P(base + 8), 4, p, p, None) == 2
    assert lib.moe_b200_quantize_hidden(p, 0, p, p, None) == 0
    # the layer on bf16 hidden states takes no scale argument
    assert lib.moe_b200_run_bf16_hidden(p, p, 0, None, p, p, p, p, 0, 2.5, 4, p, p, big, None) == 1
    assert lib.moe_b200_run_bf16_hidden(p, p, 0, p, p, p, p, p, 0, 2.5, 4, p, p, 16, None) == 3
    assert lib.moe_b200_run_bf16_hidden(p, p, 0, p, p, p, p, p, 0, 2.5, 0, p, p, 16, None) == 0


def test_ep_and_ipc_entry_points_reject_bad_arguments_without_a_device(lib):
    """The expert-parallel combine, its IPC buffer helpers and the
    allocation-free status reader check their arguments before any CUDA call."""
    P = ctypes.c_void_p
    buf = ctypes.create_string_buffer(4096 + 256)
    base = (ctypes.addressof(buf) + 255) // 256 * 256
    p = P(base)
    arr = (P * 8)(*([p] * 8))
    # shards: world * shards_per_rank must stay within 8, rank inside [0, world)
    assert lib.moe_b200_ep_combine_shards(arr, 0, arr, 0, 2, 4, p, None) == 1
    assert lib.moe_b200_ep_combine_shards(arr, 3, arr, 0, 4, 4, p, None) == 1
    assert lib.moe_b200_ep_combine_shards(arr, 1, arr, 2, 2, 4, p, None) == 1
    assert lib.moe_b200_ep_combine_shards(arr, 1, arr, 0, 9, 4, p, None) == 1
    assert lib.moe_b200_ep_combine_shards(None, 1, arr, 0, 2, 4, p, None) == 1
    assert lib.moe_b200_ep_combine_shards(arr, 4, arr, 0, 2, -1, p, None) == 1
    assert lib.moe_b200_ep_combine_shards(arr, 4, arr, 0, 2, 4, P(base + 8), None) == 2    # misaligned output
    mis = (P * 8)(*([P(base + 16)] * 8))
    assert lib.moe_b200_ep_combine_shards(mis, 4, arr, 0, 2, 4, p, None) == 2            # misaligned workspace
    assert lib.moe_b200_ep_combine_shards(arr, 4, mis, 0, 2, 4, p, None) == 2            # misaligned area
    assert lib.moe_b200_ep_combine_shards(arr, 4, arr, 0, 2, 0, p, None) == 0            # T = 0 is a no-op
    assert lib.moe_b200_ep_combine(arr, arr, 0, 2, 0, p, None) == 0
    # counter block, flagged-line buffers (72 rows of 3584 fp32 lines, 64 rows
    # of 1792 bf16 lines, 16 bytes each), then the bf16 staging rows
    lines = 72 * 3584 * 16 + 64 * 1792 * 16
    assert lib.moe_b200_ep_area_bytes(16) == 256 + lines + (16 * 7168 * 2 + 255) // 256 * 256
    assert lib.moe_b200_ep_area_bytes(-1) == 0
    out = P()
    assert lib.moe_b200_ep_buffer_alloc(0, ctypes.byref(out)) == 1
    assert lib.moe_b200_ep_buffer_alloc(16, None) == 1
    assert lib.moe_b200_ep_buffer_free(None) == 0
    assert lib.moe_b200_ipc_get_handle(None, p) == 1
    assert lib.moe_b200_ipc_get_handle(p, None) == 1
    assert lib.moe_b200_ipc_open_handle(None, ctypes.byref(out)) == 1
    assert lib.moe_b200_ipc_open_handle(p, None) == 1
    assert lib.moe_b200_ipc_close_handle(None) == 0
    assert lib.moe_b200_noalloc_read_status(None, None) == 1


def test_token_parallel_entry_points_reject_bad_arguments_without_a_device(lib):
    """The routed layer and the all-to-all entry points check their arguments
    before any CUDA call."""
    P = ctypes.c_void_p
    buf = ctypes.create_string_buffer(4096 + 256)
    base = (ctypes.addressof(buf) + 255) // 256 * 256
    p = P(base)
    big = 1 << 40
    # the routed layer: given ids and weights are required, top_k 1..8
    assert lib.moe_b200_run_routed(None, p, 1, p, p, p, p, p, p, 0, 4, p, p, big, None) == 1
    assert lib.moe_b200_run_routed(p, None, 1, p, p, p, p, p, p, 0, 4, p, p, big, None) == 1
    assert lib.moe_b200_run_routed(p, p, 0, p, p, p, p, p, p, 0, 4, p, p, big, None) == 1
    assert lib.moe_b200_run_routed(p, p, 9, p, p, p, p, p, p, 0, 4, p, p, big, None) == 1
    assert lib.moe_b200_run_routed(P(base + 2), p, 1, p, p, p, p, p, p, 0, 4, p, p, big, None) == 2
    assert lib.moe_b200_run_routed(p, p, 1, p, p, p, p, p, p, 0, 4, p, p, 16, None) == 3
    assert lib.moe_b200_run_routed(p, p, 1, p, p, p, p, p, p, 0, 0, p, p, 16, None) == 0
    # the given-routing rule is not one of the public routing methods
    assert lib.moe_b200_route_method(6, 1, p, p, 0, 4, 1.0, p, p, None) == 1
    assert lib.moe_b200_run_routing(6, 1, p, p, 0, p, p, p, p, p, p, 0, 1.0, 4, p, p, big, None) == 1
    # all-to-all: world x shards must cover the 8 shards, sizes in range
    arr = (P * 8)(*([p] * 8))
    assert lib.moe_b200_a2a_area_bytes(16, 128) > 512
    assert lib.moe_b200_a2a_area_bytes(16, 0) == 0
    assert lib.moe_b200_a2a_area_bytes(-1, 128) == 0
    assert lib.moe_b200_a2a_dispatch(p, p, p, p, 4, 16, 128, arr, 0, 2, 2, None) == 1    # 2 x 2 != 8
    assert lib.moe_b200_a2a_dispatch(p, p, p, p, 17, 16, 128, arr, 0, 2, 4, None) == 1   # T > max_tokens
    assert lib.moe_b200_a2a_dispatch(p, p, p, p, 4, 16, 128, arr, 2, 2, 4, None) == 1    # rank out of range
    assert lib.moe_b200_a2a_dispatch(None, p, p, p, 4, 16, 128, arr, 0, 2, 4, None) == 1
    assert lib.moe_b200_a2a_dispatch(p, p, P(base + 8), p, 4, 16, 128, arr, 0, 2, 4, None) == 2
    mis = (P * 8)(*([P(base + 16)] * 8))
    assert lib.moe_b200_a2a_dispatch(p, p, p, p, 4, 16, 128, mis, 0, 2, 4, None) == 2
    assert lib.moe_b200_a2a_combine(p, arr, arr, 0, 2, 4, 4, 16, 128, P(base + 8), None) == 2
    assert lib.moe_b200_a2a_combine(p, None, arr, 0, 2, 4, 4, 16, 128, p, None) == 1
    assert lib.moe_b200_a2a_combine(p, arr, arr, 0, 8, 2, 4, 16, 128, p, None) == 1     # 8 x 2 != 8
    assert lib.moe_b200_a2a_read_status(None, None, None, None) == 1
