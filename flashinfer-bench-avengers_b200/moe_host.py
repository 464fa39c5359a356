"""Host side of the B200 MoE layer: argument checks, workspace management
and the ctypes binding of libmoe_b200.so (C ABI in include/moe_b200.h).

PyTorch is used only for device memory and the current stream; all
computation runs in the library's sm_100a kernels. There is no CPU or
framework fallback: if the library is missing or the device is not an
sm_100 GPU, the calls raise.

Argument checks mirror the reference's TORCH_CHECKs
(solution/cuda/main.cpp:25-40) and raise RuntimeError like they do.
"""
from __future__ import annotations

import ctypes
import os
import threading

import torch

H = 7168
I = 2048
E_GLOBAL = 256
E_LOCAL = 32
TOP_K = 8
HIDDEN_BLOCKS = H // 128
INTER_BLOCKS = I // 128
GEMM1_OUT_BLOCKS = 2 * I // 128
MAX_TOKENS = 262144
# Calls with at least this many tokens run the token-major prefill GEMMs
# (kTokenMajorMinTokens, moe_capi.cu).
TOKEN_MAJOR_MIN_TOKENS = 512
# Sizes of the counter blocks at the start of an EP area and of an
# all-to-all area (MOE_B200_EP_COUNTER_BYTES, MOE_B200_A2A_COUNTER_BYTES).
EP_COUNTER_BYTES = 256
A2A_COUNTER_BYTES = 512

BIAS_BF16 = 0
BIAS_FP32 = 1

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libmoe_b200.so")

_lib = None
_lib_lock = threading.Lock()

_P = ctypes.c_void_p
_I64 = ctypes.c_int64


class WorkspaceLayout(ctypes.Structure):
    _fields_ = [
        ("total_bytes", ctypes.c_size_t),
        ("counts", ctypes.c_size_t),
        ("status", ctypes.c_size_t),
        ("seg_off", ctypes.c_size_t),
        ("topk_idx", ctypes.c_size_t),
        ("topk_w", ctypes.c_size_t),
        ("perm_tok", ctypes.c_size_t),
        ("perm_w", ctypes.c_size_t),
        ("a_perm", ctypes.c_size_t),
        ("sa_perm", ctypes.c_size_t),
        ("c_hi", ctypes.c_size_t),
        ("c_lo", ctypes.c_size_t),
        ("c_scale", ctypes.c_size_t),
        ("y_acc", ctypes.c_size_t),
        ("g1_acc", ctypes.c_size_t),
        ("cap_rows", ctypes.c_int64),
        ("chunk_counts", ctypes.c_size_t),
        ("sched", ctypes.c_size_t),
        ("perm_row", ctypes.c_size_t),
        ("tok_slot", ctypes.c_size_t),
        ("n_touched", ctypes.c_size_t),
        ("slot_tok", ctypes.c_size_t),
        ("hidden_q", ctypes.c_size_t),
        ("hidden_qs", ctypes.c_size_t),
    ]


class A2aLayout(ctypes.Structure):
    _fields_ = [
        ("total_bytes", ctypes.c_size_t),
        ("send_slot", ctypes.c_size_t),
        ("dest_row", ctypes.c_size_t),
        ("slab_idx", ctypes.c_size_t),
        ("slab_w", ctypes.c_size_t),
        ("slab_scale", ctypes.c_size_t),
        ("slab_rows", ctypes.c_size_t),
    ]


def _build_module():
    """This package's build.py, loaded by path (a top-level module named
    ``build`` could be another package's)."""
    import importlib.util

    spec = importlib.util.spec_from_file_location("moe_b200_build", os.path.join(_HERE, "build.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def load_library(path: str = LIB_PATH) -> ctypes.CDLL:
    """Loads (once) the C-ABI library. The in-tree library is first compiled
    from csrc/ when it is missing or older than its sources (nvcc needed);
    a build failure raises, since the layer has no fallback implementation."""
    global _lib
    with _lib_lock:
        if _lib is not None:
            return _lib
        if os.path.abspath(path) == os.path.abspath(LIB_PATH):
            _build_module().build()
        if not os.path.exists(path):
            raise RuntimeError(f"{path} is missing (the MoE layer has no fallback implementation)")
        lib = ctypes.CDLL(path)
        lib.moe_b200_workspace_bytes.argtypes = [_I64]
        lib.moe_b200_workspace_bytes.restype = ctypes.c_size_t
        lib.moe_b200_run.argtypes = [_P, _P, ctypes.c_int, _P, _P, _P, _P, _P, _P, _I64,
                                     ctypes.c_double, _I64, _P, _P, ctypes.c_size_t, _P]
        lib.moe_b200_run.restype = ctypes.c_int
        lib.moe_b200_run_bf16_hidden.argtypes = [_P, _P, ctypes.c_int, _P, _P, _P, _P, _P, _I64,
                                                 ctypes.c_double, _I64, _P, _P, ctypes.c_size_t, _P]
        lib.moe_b200_run_bf16_hidden.restype = ctypes.c_int
        lib.moe_b200_quantize_hidden.argtypes = [_P, _I64, _P, _P, _P]
        lib.moe_b200_quantize_hidden.restype = ctypes.c_int
        lib.moe_b200_run_routing.argtypes = [ctypes.c_int, ctypes.c_int, _P, _P, ctypes.c_int, _P, _P, _P, _P, _P,
                                             _P, _I64, ctypes.c_double, _I64, _P, _P, ctypes.c_size_t, _P]
        lib.moe_b200_run_routing.restype = ctypes.c_int
        lib.moe_b200_route_method.argtypes = [ctypes.c_int, ctypes.c_int, _P, _P, ctypes.c_int, _I64,
                                              ctypes.c_double, _P, _P, _P]
        lib.moe_b200_route_method.restype = ctypes.c_int
        lib.moe_b200_route.argtypes = [_P, _P, ctypes.c_int, _I64, ctypes.c_double, _P, _P, _P]
        lib.moe_b200_route.restype = ctypes.c_int
        lib.moe_b200_read_status.argtypes = [_P, ctypes.POINTER(ctypes.c_uint32), _P]
        lib.moe_b200_read_status.restype = ctypes.c_int
        lib.moe_b200_status_string.argtypes = [ctypes.c_int]
        lib.moe_b200_status_string.restype = ctypes.c_char_p
        lib.moe_b200_get_workspace_layout.argtypes = [_I64, ctypes.POINTER(WorkspaceLayout)]
        lib.moe_b200_get_workspace_layout.restype = ctypes.c_int
        lib.moe_b200_set_stage_events.argtypes = [ctypes.POINTER(ctypes.c_void_p), ctypes.c_int]
        lib.moe_b200_set_stage_events.restype = ctypes.c_int
        lib.moe_b200_abi_version.argtypes = []
        lib.moe_b200_abi_version.restype = ctypes.c_int
        lib.moe_b200_ep_area_bytes.argtypes = [_I64]
        lib.moe_b200_ep_area_bytes.restype = ctypes.c_size_t
        lib.moe_b200_ep_combine.argtypes = [ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(ctypes.c_void_p),
                                            ctypes.c_int, ctypes.c_int, _I64, _P, _P]
        lib.moe_b200_ep_combine.restype = ctypes.c_int
        lib.moe_b200_ep_combine_shards.argtypes = [ctypes.POINTER(ctypes.c_void_p), ctypes.c_int,
                                                   ctypes.POINTER(ctypes.c_void_p), ctypes.c_int, ctypes.c_int,
                                                   _I64, _P, _P]
        lib.moe_b200_ep_combine_shards.restype = ctypes.c_int
        lib.moe_b200_ep_buffer_alloc.argtypes = [ctypes.c_size_t, ctypes.POINTER(ctypes.c_void_p)]
        lib.moe_b200_ep_buffer_alloc.restype = ctypes.c_int
        lib.moe_b200_ep_buffer_free.argtypes = [_P]
        lib.moe_b200_ep_buffer_free.restype = ctypes.c_int
        lib.moe_b200_ipc_get_handle.argtypes = [_P, _P]
        lib.moe_b200_ipc_get_handle.restype = ctypes.c_int
        lib.moe_b200_ipc_open_handle.argtypes = [_P, ctypes.POINTER(ctypes.c_void_p)]
        lib.moe_b200_ipc_open_handle.restype = ctypes.c_int
        lib.moe_b200_ipc_close_handle.argtypes = [_P]
        lib.moe_b200_ipc_close_handle.restype = ctypes.c_int
        lib.moe_b200_run_noalloc.argtypes = [_P, _P, ctypes.c_int, _P, _P, _P, _P, _P, _P, _I64,
                                             ctypes.c_double, _I64, _P, _P]
        lib.moe_b200_run_noalloc.restype = ctypes.c_int
        lib.moe_b200_noalloc_read_status.argtypes = [ctypes.POINTER(ctypes.c_uint32), _P]
        lib.moe_b200_noalloc_read_status.restype = ctypes.c_int
        lib.moe_b200_run_routed.argtypes = [_P, _P, ctypes.c_int, _P, _P, _P, _P, _P, _P, _I64, _I64, _P, _P,
                                            ctypes.c_size_t, _P]
        lib.moe_b200_run_routed.restype = ctypes.c_int
        lib.moe_b200_routed_workspace_bytes.argtypes = [_I64, ctypes.c_int]
        lib.moe_b200_routed_workspace_bytes.restype = ctypes.c_size_t
        lib.moe_b200_get_routed_workspace_layout.argtypes = [_I64, ctypes.c_int, ctypes.POINTER(WorkspaceLayout)]
        lib.moe_b200_get_routed_workspace_layout.restype = ctypes.c_int
        lib.moe_b200_a2a_area_bytes.argtypes = [_I64, _I64]
        lib.moe_b200_a2a_area_bytes.restype = ctypes.c_size_t
        lib.moe_b200_a2a_get_layout.argtypes = [_I64, _I64, ctypes.POINTER(A2aLayout)]
        lib.moe_b200_a2a_get_layout.restype = ctypes.c_int
        lib.moe_b200_a2a_dispatch.argtypes = [_P, _P, _P, _P, _I64, _I64, _I64, ctypes.POINTER(ctypes.c_void_p),
                                              ctypes.c_int, ctypes.c_int, ctypes.c_int, _P]
        lib.moe_b200_a2a_dispatch.restype = ctypes.c_int
        lib.moe_b200_a2a_combine.argtypes = [_P, ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(ctypes.c_void_p),
                                             ctypes.c_int, ctypes.c_int, ctypes.c_int, _I64, _I64, _I64, _P, _P]
        lib.moe_b200_a2a_combine.restype = ctypes.c_int
        lib.moe_b200_a2a_read_status.argtypes = [_P, ctypes.POINTER(ctypes.c_uint32), ctypes.POINTER(ctypes.c_int32),
                                                 _P]
        lib.moe_b200_a2a_read_status.restype = ctypes.c_int
        _lib = lib
        return lib


def status_string(code: int) -> str:
    return load_library().moe_b200_status_string(int(code)).decode()


def _raise_on(code: int, what: str) -> None:
    if code != 0:
        raise RuntimeError(f"{what} failed: {status_string(code)} (status {code})")


def workspace_bytes(num_tokens: int) -> int:
    return int(load_library().moe_b200_workspace_bytes(int(num_tokens)))


def routed_workspace_bytes(num_tokens: int, top_k: int) -> int:
    """Workspace of moe_b200_run_routed for T tokens of at most top_k picks."""
    return int(load_library().moe_b200_routed_workspace_bytes(int(num_tokens), int(top_k)))


def routed_workspace_layout(num_tokens: int, top_k: int) -> WorkspaceLayout:
    out = WorkspaceLayout()
    _raise_on(load_library().moe_b200_get_routed_workspace_layout(int(num_tokens), int(top_k), ctypes.byref(out)),
              "moe_b200_get_routed_workspace_layout")
    return out


def workspace_layout(num_tokens: int) -> WorkspaceLayout:
    out = WorkspaceLayout()
    _raise_on(load_library().moe_b200_get_workspace_layout(int(num_tokens), ctypes.byref(out)),
              "moe_b200_get_workspace_layout")
    return out


# One cached workspace per device; it only grows. Calls on the same device
# and stream reuse it, which is what stream ordering makes safe.
_workspaces: dict[int, torch.Tensor] = {}
_ws_lock = threading.Lock()


def get_workspace(num_tokens: int, device: torch.device) -> torch.Tensor:
    need = workspace_bytes(num_tokens)
    idx = device.index if device.index is not None else torch.cuda.current_device()
    with _ws_lock:
        ws = _workspaces.get(idx)
        if ws is None or ws.numel() < need:
            ws = torch.empty(max(need, 1 << 20), dtype=torch.uint8, device=torch.device("cuda", idx))
            _workspaces[idx] = ws
        return ws


def _check(cond: bool, msg: str) -> None:
    if not cond:
        raise RuntimeError(msg)


def _check_same_cuda_device(**tensors) -> None:
    """Every tensor is a CUDA tensor on the first one's device (the kernels
    dereference their pointers on that device)."""
    dev = None
    for name, t in tensors.items():
        _check(isinstance(t, torch.Tensor) and t.is_cuda, f"{name} must be a CUDA tensor")
        dev = t.device if dev is None else dev
        _check(t.device == dev, f"{name} must be on {dev}")


def _check_inputs(routing_logits, routing_bias, hidden_states, hidden_states_scale, gemm1_weights,
                  gemm1_weights_scale, gemm2_weights, gemm2_weights_scale) -> int:
    """Checks the layer inputs; hidden_states_scale None means bf16 hidden
    states (run_bf16_hidden) instead of e4m3 ones with their scales."""
    bf16_hidden = hidden_states_scale is None
    tensors = {
        "routing_logits": routing_logits,
        "routing_bias": routing_bias,
        "hidden_states": hidden_states,
        "hidden_states_scale": hidden_states_scale,
        "gemm1_weights": gemm1_weights,
        "gemm1_weights_scale": gemm1_weights_scale,
        "gemm2_weights": gemm2_weights,
        "gemm2_weights_scale": gemm2_weights_scale,
    }
    if bf16_hidden:
        del tensors["hidden_states_scale"]
    if routing_bias is None:   # other routing methods may run without a bias
        del tensors["routing_bias"]
    for name, t in tensors.items():
        _check(isinstance(t, torch.Tensor), f"{name} must be a torch.Tensor")
        _check(t.is_cuda, f"{name} must be CUDA")
    dev = routing_logits.device
    for name, t in tensors.items():
        _check(t.device == dev, f"{name} must be on {dev}")
    _check(routing_logits.dim() == 2 and routing_logits.size(1) == E_GLOBAL,
           f"routing_logits must be [T, {E_GLOBAL}]")
    T = routing_logits.size(0)
    _check(T <= MAX_TOKENS, f"at most {MAX_TOKENS} tokens per call")
    _check(routing_logits.dtype == torch.float32, "routing_logits must be float32")
    _check(routing_bias is None or routing_bias.numel() == E_GLOBAL, f"routing_bias must have {E_GLOBAL} elements")
    _check(tuple(hidden_states.shape) == (T, H), f"hidden_states must be [T, {H}]")
    if bf16_hidden:
        _check(hidden_states.dtype == torch.bfloat16, "hidden_states must be bfloat16")
    else:
        _check(hidden_states.dtype == torch.float8_e4m3fn, "hidden_states must be float8_e4m3fn")
        _check(tuple(hidden_states_scale.shape) == (HIDDEN_BLOCKS, T),
               f"hidden_states_scale must be [{HIDDEN_BLOCKS}, T]")
        _check(hidden_states_scale.dtype == torch.float32, "hidden_states_scale must be float32")
    _check(tuple(gemm1_weights.shape) == (E_LOCAL, 2 * I, H), f"gemm1_weights must be [{E_LOCAL}, {2 * I}, {H}]")
    _check(gemm1_weights.dtype == torch.float8_e4m3fn, "gemm1_weights must be float8_e4m3fn")
    _check(tuple(gemm1_weights_scale.shape) == (E_LOCAL, GEMM1_OUT_BLOCKS, HIDDEN_BLOCKS),
           f"gemm1_weights_scale must be [{E_LOCAL}, {GEMM1_OUT_BLOCKS}, {HIDDEN_BLOCKS}]")
    _check(gemm1_weights_scale.dtype == torch.float32, "gemm1_weights_scale must be float32")
    _check(tuple(gemm2_weights.shape) == (E_LOCAL, H, I), f"gemm2_weights must be [{E_LOCAL}, {H}, {I}]")
    _check(gemm2_weights.dtype == torch.float8_e4m3fn, "gemm2_weights must be float8_e4m3fn")
    _check(tuple(gemm2_weights_scale.shape) == (E_LOCAL, HIDDEN_BLOCKS, INTER_BLOCKS),
           f"gemm2_weights_scale must be [{E_LOCAL}, {HIDDEN_BLOCKS}, {INTER_BLOCKS}]")
    _check(gemm2_weights_scale.dtype == torch.float32, "gemm2_weights_scale must be float32")
    for name in ("hidden_states", "gemm1_weights", "gemm2_weights"):
        _check(tensors[name].is_contiguous(), f"{name} must be contiguous")
    return T


def _bias_arg(routing_bias: torch.Tensor | None) -> tuple[torch.Tensor | None, int]:
    if routing_bias is None:
        return None, BIAS_BF16
    b = routing_bias.reshape(-1)
    if b.dtype == torch.bfloat16:
        return b.contiguous(), BIAS_BF16
    return b.to(torch.float32).contiguous(), BIAS_FP32


def run_dps(routing_logits, routing_bias, hidden_states, hidden_states_scale, gemm1_weights,
            gemm1_weights_scale, gemm2_weights, gemm2_weights_scale, local_expert_offset,
            routed_scaling_factor, output, workspace: torch.Tensor | None = None) -> torch.Tensor:
    """Destination-passing form: writes the bf16 [T, 7168] result into ``output``.

    ``output=None`` (with an explicit ``workspace``) leaves the fp32 combine
    rows in the workspace for ep_combine and writes no output."""
    T = _check_inputs(routing_logits, routing_bias, hidden_states, hidden_states_scale,
                      gemm1_weights, gemm1_weights_scale, gemm2_weights, gemm2_weights_scale)
    if output is None:
        _check(workspace is not None, "output=None needs an explicit workspace")
    else:
        _check(isinstance(output, torch.Tensor) and output.device == routing_logits.device,
               "output must be a CUDA tensor on the inputs' device")
        _check(tuple(output.shape) == (T, H) and output.dtype == torch.bfloat16 and output.is_contiguous(),
               f"output must be a contiguous bf16 [T, {H}] tensor")
    if T == 0:
        return output
    lib = load_library()
    dev = routing_logits.device
    with torch.cuda.device(dev):
        logits = routing_logits.contiguous()
        bias, bias_dtype = _bias_arg(routing_bias)
        hs_scale = hidden_states_scale.contiguous()
        s13 = gemm1_weights_scale.contiguous()
        s2 = gemm2_weights_scale.contiguous()
        ws = workspace if workspace is not None else get_workspace(T, dev)
        stream = torch.cuda.current_stream(dev).cuda_stream
        code = lib.moe_b200_run(
            logits.data_ptr(), bias.data_ptr(), bias_dtype, hidden_states.data_ptr(),
            hs_scale.data_ptr(), gemm1_weights.data_ptr(), s13.data_ptr(), gemm2_weights.data_ptr(),
            s2.data_ptr(), int(local_expert_offset), float(routed_scaling_factor), T,
            output.data_ptr() if output is not None else None, ws.data_ptr(), ws.numel(), stream)
    _raise_on(code, "moe_b200_run")
    return output


def run_bf16_hidden(routing_logits, routing_bias, hidden_states, gemm1_weights, gemm1_weights_scale,
                    gemm2_weights, gemm2_weights_scale, local_expert_offset, routed_scaling_factor,
                    output: torch.Tensor | None = None, workspace: torch.Tensor | None = None) -> torch.Tensor:
    """The layer on bf16 hidden states [T, 7168]: each (token, expert) row is
    quantised (quantize_hidden's convention) while it is copied into the
    permuted buffers (moe_b200_run_bf16_hidden). Returns ``output`` (allocated
    when None)."""
    T = _check_inputs(routing_logits, routing_bias, hidden_states, None,
                      gemm1_weights, gemm1_weights_scale, gemm2_weights, gemm2_weights_scale)
    dev = routing_logits.device
    if output is None:
        output = torch.empty((T, H), dtype=torch.bfloat16, device=dev)
    _check(isinstance(output, torch.Tensor) and output.device == dev and tuple(output.shape) == (T, H)
           and output.dtype == torch.bfloat16 and output.is_contiguous(),
           f"output must be a contiguous bf16 [T, {H}] tensor on the inputs' device")
    if T == 0:
        return output
    lib = load_library()
    with torch.cuda.device(dev):
        logits = routing_logits.contiguous()
        bias, bias_dtype = _bias_arg(routing_bias)
        s13 = gemm1_weights_scale.contiguous()
        s2 = gemm2_weights_scale.contiguous()
        ws = workspace if workspace is not None else get_workspace(T, dev)
        code = lib.moe_b200_run_bf16_hidden(
            logits.data_ptr(), bias.data_ptr(), bias_dtype, hidden_states.data_ptr(), gemm1_weights.data_ptr(),
            s13.data_ptr(), gemm2_weights.data_ptr(), s2.data_ptr(), int(local_expert_offset),
            float(routed_scaling_factor), T, output.data_ptr(), ws.data_ptr(), ws.numel(),
            torch.cuda.current_stream(dev).cuda_stream)
    _raise_on(code, "moe_b200_run_bf16_hidden")
    return output


# Routing methods, numbered as flashinfer's RoutingMethodType (moe_b200.h).
ROUTING_DEFAULT, ROUTING_RENORMALIZE, ROUTING_DEEPSEEK_V3 = 0, 1, 2
ROUTING_LLAMA4, ROUTING_RENORMALIZE_NAIVE, ROUTING_TOPK = 3, 4, 5


def run_routing(routing_method: int, top_k: int, routing_logits, routing_bias, hidden_states, hidden_states_scale,
                gemm1_weights, gemm1_weights_scale, gemm2_weights, gemm2_weights_scale, local_expert_offset,
                routed_scaling_factor, output: torch.Tensor | None = None,
                workspace: torch.Tensor | None = None) -> torch.Tensor:
    """The layer with another routing method of the family ahead of the same
    permutation and GEMMs (moe_b200_run_routing); routing_bias may be None
    except for ROUTING_DEEPSEEK_V3. Returns ``output`` (allocated when None)."""
    T = _check_inputs(routing_logits, routing_bias, hidden_states, hidden_states_scale,
                      gemm1_weights, gemm1_weights_scale, gemm2_weights, gemm2_weights_scale)
    dev = routing_logits.device
    if output is None:
        output = torch.empty((T, H), dtype=torch.bfloat16, device=dev)
    _check(isinstance(output, torch.Tensor) and output.device == dev and tuple(output.shape) == (T, H)
           and output.dtype == torch.bfloat16 and output.is_contiguous(),
           f"output must be a contiguous bf16 [T, {H}] tensor on the inputs' device")
    if T == 0:
        return output
    lib = load_library()
    with torch.cuda.device(dev):
        logits = routing_logits.contiguous()
        bias, bias_dtype = _bias_arg(routing_bias)
        hs_scale = hidden_states_scale.contiguous()
        s13 = gemm1_weights_scale.contiguous()
        s2 = gemm2_weights_scale.contiguous()
        ws = workspace if workspace is not None else get_workspace(T, dev)
        code = lib.moe_b200_run_routing(
            int(routing_method), int(top_k), logits.data_ptr(), bias.data_ptr() if bias is not None else None,
            bias_dtype, hidden_states.data_ptr(), hs_scale.data_ptr(), gemm1_weights.data_ptr(), s13.data_ptr(),
            gemm2_weights.data_ptr(), s2.data_ptr(), int(local_expert_offset), float(routed_scaling_factor), T,
            output.data_ptr(), ws.data_ptr(), ws.numel(), torch.cuda.current_stream(dev).cuda_stream)
    _raise_on(code, "moe_b200_run_routing")
    return output


def route_method(routing_method: int, top_k: int, routing_logits, routing_bias,
                 routed_scaling_factor) -> tuple[torch.Tensor, torch.Tensor]:
    """Routing only, any method of the family: (topk_idx int32 [T, 8] best
    first, -(1 << 30) after top_k; topk_w fp32 [T, 8], 0 after top_k)."""
    _check(routing_logits.is_cuda and routing_logits.dtype == torch.float32
           and routing_logits.dim() == 2 and routing_logits.size(1) == E_GLOBAL,
           f"routing_logits must be a CUDA float32 [T, {E_GLOBAL}] tensor")
    T = routing_logits.size(0)
    dev = routing_logits.device
    idx = torch.empty((T, TOP_K), dtype=torch.int32, device=dev)
    w = torch.empty((T, TOP_K), dtype=torch.float32, device=dev)
    if T == 0:
        return idx, w
    lib = load_library()
    with torch.cuda.device(dev):
        logits = routing_logits.contiguous()
        bias, bias_dtype = _bias_arg(routing_bias.to(dev) if routing_bias is not None else None)
        code = lib.moe_b200_route_method(int(routing_method), int(top_k), logits.data_ptr(),
                                         bias.data_ptr() if bias is not None else None, bias_dtype, T,
                                         float(routed_scaling_factor), idx.data_ptr(), w.data_ptr(),
                                         torch.cuda.current_stream(dev).cuda_stream)
    _raise_on(code, "moe_b200_route_method")
    return idx, w


def quantize_hidden(hidden_states: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """bf16 [T, 7168] -> (e4m3 [T, 7168], fp32 block scales [56, T]): per
    128-column block scale = amax / 448 (1 for an all-zero block), value =
    e4m3(x / scale) (moe_b200_quantize_hidden)."""
    _check(isinstance(hidden_states, torch.Tensor) and hidden_states.is_cuda
           and hidden_states.dtype == torch.bfloat16 and hidden_states.dim() == 2
           and hidden_states.size(1) == H, f"hidden_states must be a CUDA bf16 [T, {H}] tensor")
    T = hidden_states.size(0)
    _check(T <= MAX_TOKENS, f"at most {MAX_TOKENS} tokens per call")
    dev = hidden_states.device
    q = torch.empty((T, H), dtype=torch.float8_e4m3fn, device=dev)
    s = torch.empty((HIDDEN_BLOCKS, T), dtype=torch.float32, device=dev)
    if T == 0:
        return q, s
    with torch.cuda.device(dev):
        x = hidden_states.contiguous()
        code = load_library().moe_b200_quantize_hidden(x.data_ptr(), T, q.data_ptr(), s.data_ptr(),
                                                        torch.cuda.current_stream(dev).cuda_stream)
    _raise_on(code, "moe_b200_quantize_hidden")
    return q, s


def ep_area_bytes(num_tokens: int) -> int:
    """EP area of one rank (counters + bf16 staging) for moe_b200_ep_combine."""
    return int(load_library().moe_b200_ep_area_bytes(int(num_tokens)))


def ep_combine(rank_workspace_ptrs: list[int], rank_area_ptrs: list[int], rank: int, num_tokens: int,
               output: torch.Tensor) -> torch.Tensor:
    """bf16 sum over the ranks of their layer outputs into ``output`` (see
    moe_b200_ep_combine); ``rank_workspace_ptrs[q]`` / ``rank_area_ptrs[q]``
    are rank q's workspace and EP area addresses in this process."""
    _check(output.is_cuda and output.dtype == torch.bfloat16 and output.is_contiguous()
           and tuple(output.shape) == (int(num_tokens), H), f"output must be a contiguous bf16 [T, {H}] tensor")
    world = len(rank_workspace_ptrs)
    _check(len(rank_area_ptrs) == world, "one EP area per rank")
    ws = (ctypes.c_void_p * world)(*[ctypes.c_void_p(int(p)) for p in rank_workspace_ptrs])
    areas = (ctypes.c_void_p * world)(*[ctypes.c_void_p(int(p)) for p in rank_area_ptrs])
    stream = torch.cuda.current_stream(output.device).cuda_stream
    _raise_on(load_library().moe_b200_ep_combine(ws, areas, int(rank), world, int(num_tokens),
                                                   output.data_ptr(), stream), "moe_b200_ep_combine")
    return output


def ep_combine_shards(shard_workspace_ptrs: list[int], shards_per_rank: int, rank_area_ptrs: list[int],
                      rank: int, num_tokens: int, output: torch.Tensor) -> torch.Tensor:
    """moe_b200_ep_combine_shards: bf16 sum over every shard of every rank
    into ``output``; ``shard_workspace_ptrs`` lists world * shards_per_rank
    workspace addresses rank-major, ``rank_area_ptrs`` one EP area per rank."""
    _check(output.is_cuda and output.dtype == torch.bfloat16 and output.is_contiguous()
           and tuple(output.shape) == (int(num_tokens), H), f"output must be a contiguous bf16 [T, {H}] tensor")
    world = len(rank_area_ptrs)
    _check(len(shard_workspace_ptrs) == world * int(shards_per_rank), "world * shards_per_rank workspaces")
    n = len(shard_workspace_ptrs)
    ws = (ctypes.c_void_p * n)(*[ctypes.c_void_p(int(p)) for p in shard_workspace_ptrs])
    areas = (ctypes.c_void_p * world)(*[ctypes.c_void_p(int(p)) for p in rank_area_ptrs])
    stream = torch.cuda.current_stream(output.device).cuda_stream
    _raise_on(load_library().moe_b200_ep_combine_shards(ws, int(shards_per_rank), areas, int(rank), world,
                                                          int(num_tokens), output.data_ptr(), stream),
              "moe_b200_ep_combine_shards")
    return output


def run_routed_ptrs(topk_idx_ptr: int, topk_w_ptr: int, top_k: int, hidden_ptr: int, hidden_scale_ptr: int,
                    gemm1_weights, gemm1_weights_scale, gemm2_weights, gemm2_weights_scale, local_expert_offset: int,
                    num_tokens: int, workspace: torch.Tensor, output: torch.Tensor | None = None) -> None:
    """moe_b200_run_routed on device pointers (the rows of an all-to-all
    receive slab): routing given as [T, top_k] ids / weights; with
    ``output=None`` the fp32 combine rows stay in ``workspace``."""
    for name, t, shape, dt in (("gemm1_weights", gemm1_weights, (E_LOCAL, 2 * I, H), torch.float8_e4m3fn),
                               ("gemm1_weights_scale", gemm1_weights_scale, (E_LOCAL, GEMM1_OUT_BLOCKS, HIDDEN_BLOCKS),
                                torch.float32),
                               ("gemm2_weights", gemm2_weights, (E_LOCAL, H, I), torch.float8_e4m3fn),
                               ("gemm2_weights_scale", gemm2_weights_scale, (E_LOCAL, HIDDEN_BLOCKS, INTER_BLOCKS),
                                torch.float32)):
        _check(isinstance(t, torch.Tensor) and t.is_cuda and tuple(t.shape) == shape and t.dtype == dt
               and t.is_contiguous(), f"{name} must be a contiguous CUDA {dt} tensor of shape {shape}")
    _check_same_cuda_device(gemm1_weights=gemm1_weights, gemm1_weights_scale=gemm1_weights_scale,
                            gemm2_weights=gemm2_weights, gemm2_weights_scale=gemm2_weights_scale,
                            workspace=workspace, **({"output": output} if output is not None else {}))
    if output is not None:
        _check(output.dtype == torch.bfloat16 and tuple(output.shape) == (int(num_tokens), H)
               and output.is_contiguous(), f"output must be a contiguous bf16 [T, {H}] tensor")
    dev = gemm1_weights.device
    with torch.cuda.device(dev):
        code = load_library().moe_b200_run_routed(
            int(topk_idx_ptr), int(topk_w_ptr), int(top_k), int(hidden_ptr), int(hidden_scale_ptr),
            gemm1_weights.data_ptr(), gemm1_weights_scale.data_ptr(), gemm2_weights.data_ptr(),
            gemm2_weights_scale.data_ptr(), int(local_expert_offset), int(num_tokens),
            output.data_ptr() if output is not None else None, workspace.data_ptr(), workspace.numel(),
            torch.cuda.current_stream(dev).cuda_stream)
    _raise_on(code, "moe_b200_run_routed")


def run_routed(topk_idx: torch.Tensor, topk_w: torch.Tensor, hidden_states, hidden_states_scale, gemm1_weights,
               gemm1_weights_scale, gemm2_weights, gemm2_weights_scale, local_expert_offset,
               output: torch.Tensor | None = None, workspace: torch.Tensor | None = None) -> torch.Tensor:
    """The layer with given routing: topk_idx int32 / topk_w fp32 [T, top_k]
    (global expert ids, final weights). Returns ``output`` (allocated when None)."""
    _check(topk_idx.is_cuda and topk_idx.dtype == torch.int32 and topk_idx.dim() == 2 and topk_idx.is_contiguous(),
           "topk_idx must be a contiguous CUDA int32 [T, top_k] tensor")
    T, k = topk_idx.shape
    _check(1 <= k <= TOP_K, f"top_k must be 1..{TOP_K}")
    _check(topk_w.is_cuda and topk_w.dtype == torch.float32 and tuple(topk_w.shape) == (T, k)
           and topk_w.is_contiguous(), "topk_w must be a contiguous CUDA float32 tensor shaped like topk_idx")
    _check(hidden_states.is_cuda and hidden_states.dtype == torch.float8_e4m3fn and tuple(hidden_states.shape) == (T, H)
           and hidden_states.is_contiguous(), f"hidden_states must be a contiguous float8_e4m3fn [T, {H}] tensor")
    hs_scale = hidden_states_scale.contiguous()
    _check(hs_scale.dtype == torch.float32 and tuple(hs_scale.shape) == (HIDDEN_BLOCKS, T),
           f"hidden_states_scale must be float32 [{HIDDEN_BLOCKS}, T]")
    dev = topk_idx.device
    if output is None:
        output = torch.empty((T, H), dtype=torch.bfloat16, device=dev)
    if T == 0:
        return output
    if workspace is None:
        workspace = torch.empty(routed_workspace_bytes(T, k), dtype=torch.uint8, device=dev)
    ws = workspace
    run_routed_ptrs(topk_idx.data_ptr(), topk_w.data_ptr(), k, hidden_states.data_ptr(), hs_scale.data_ptr(),
                    gemm1_weights, gemm1_weights_scale.contiguous(), gemm2_weights, gemm2_weights_scale.contiguous(),
                    local_expert_offset, T, ws, output)
    return output


def a2a_area_bytes(max_tokens: int, recv_capacity: int) -> int:
    return int(load_library().moe_b200_a2a_area_bytes(int(max_tokens), int(recv_capacity)))


def a2a_layout(max_tokens: int, recv_capacity: int) -> A2aLayout:
    out = A2aLayout()
    _raise_on(load_library().moe_b200_a2a_get_layout(int(max_tokens), int(recv_capacity), ctypes.byref(out)),
              "moe_b200_a2a_get_layout")
    return out


def _ptr_array(ptrs) -> ctypes.Array:
    return (ctypes.c_void_p * len(ptrs))(*[ctypes.c_void_p(int(p)) for p in ptrs])


def a2a_dispatch(topk_idx: torch.Tensor, topk_w: torch.Tensor, hidden_states: torch.Tensor,
                 hidden_states_scale: torch.Tensor, max_tokens: int, recv_capacity: int, rank_area_ptrs: list[int],
                 rank: int, shards_per_rank: int) -> None:
    """moe_b200_a2a_dispatch of this rank's T tokens (picks from moe_b200_route)."""
    _check_same_cuda_device(topk_idx=topk_idx, topk_w=topk_w, hidden_states=hidden_states,
                            hidden_states_scale=hidden_states_scale)
    T = int(hidden_states.shape[0])
    _check(tuple(topk_idx.shape) == (T, TOP_K) and topk_idx.dtype == torch.int32 and topk_idx.is_contiguous(),
           "topk_idx must be int32 [T, 8]")
    _check(tuple(topk_w.shape) == (T, TOP_K) and topk_w.dtype == torch.float32 and topk_w.is_contiguous(),
           "topk_w must be float32 [T, 8]")
    _check(hidden_states.dtype == torch.float8_e4m3fn and hidden_states.is_contiguous()
           and tuple(hidden_states.shape) == (T, H), f"hidden_states must be e4m3 [T, {H}]")
    _check(tuple(hidden_states_scale.shape) == (HIDDEN_BLOCKS, T) and hidden_states_scale.is_contiguous()
           and hidden_states_scale.dtype == torch.float32, f"hidden_states_scale must be float32 [{HIDDEN_BLOCKS}, T]")
    dev = hidden_states.device
    with torch.cuda.device(dev):
        code = load_library().moe_b200_a2a_dispatch(
            topk_idx.data_ptr(), topk_w.data_ptr(), hidden_states.data_ptr(), hidden_states_scale.data_ptr(), T,
            int(max_tokens), int(recv_capacity), _ptr_array(rank_area_ptrs), int(rank), len(rank_area_ptrs),
            int(shards_per_rank), torch.cuda.current_stream(dev).cuda_stream)
    _raise_on(code, "moe_b200_a2a_dispatch")


def a2a_combine(topk_idx: torch.Tensor, shard_workspace_ptrs: list[int], rank_area_ptrs: list[int], rank: int,
                shards_per_rank: int, max_tokens: int, recv_capacity: int, output: torch.Tensor) -> torch.Tensor:
    """moe_b200_a2a_combine into this rank's bf16 output [T, 7168]."""
    _check_same_cuda_device(topk_idx=topk_idx, output=output)
    T = int(topk_idx.shape[0])
    _check(tuple(topk_idx.shape) == (T, TOP_K) and topk_idx.dtype == torch.int32 and topk_idx.is_contiguous(),
           "topk_idx must be int32 [T, 8]")
    _check(output.is_cuda and output.dtype == torch.bfloat16 and output.is_contiguous()
           and tuple(output.shape) == (T, H), f"output must be a contiguous bf16 [T, {H}] tensor")
    dev = output.device
    with torch.cuda.device(dev):
        code = load_library().moe_b200_a2a_combine(
            topk_idx.data_ptr(), _ptr_array(shard_workspace_ptrs), _ptr_array(rank_area_ptrs), int(rank),
            len(rank_area_ptrs), int(shards_per_rank), T, int(max_tokens), int(recv_capacity), output.data_ptr(),
            torch.cuda.current_stream(dev).cuda_stream)
    _raise_on(code, "moe_b200_a2a_combine")
    return output


def a2a_read_status(area: torch.Tensor) -> tuple[int, int]:
    """(status bits, rows received) of this rank's last all-to-all call."""
    st, rows = ctypes.c_uint32(0), ctypes.c_int32(0)
    with torch.cuda.device(area.device):
        code = load_library().moe_b200_a2a_read_status(area.data_ptr(), ctypes.byref(st), ctypes.byref(rows),
                                                         torch.cuda.current_stream(area.device).cuda_stream)
    if code not in (0, 7):
        _raise_on(code, "moe_b200_a2a_read_status")
    return int(st.value), int(rows.value)


def run_noalloc(routing_logits, routing_bias, hidden_states, hidden_states_scale, gemm1_weights,
                gemm1_weights_scale, gemm2_weights, gemm2_weights_scale, local_expert_offset,
                routed_scaling_factor, output: torch.Tensor) -> torch.Tensor:
    """moe_b200_run_noalloc: the layer for at most 16 tokens with the
    library's fixed scratch array instead of a workspace."""
    T = _check_inputs(routing_logits, routing_bias, hidden_states, hidden_states_scale,
                      gemm1_weights, gemm1_weights_scale, gemm2_weights, gemm2_weights_scale)
    _check(isinstance(output, torch.Tensor) and output.device == routing_logits.device
           and tuple(output.shape) == (T, H) and output.dtype == torch.bfloat16 and output.is_contiguous(),
           f"output must be a contiguous bf16 [T, {H}] tensor on the inputs' device")
    if T == 0:
        return output
    dev = routing_logits.device
    with torch.cuda.device(dev):
        logits = routing_logits.contiguous()
        bias, bias_dtype = _bias_arg(routing_bias)
        hs_scale = hidden_states_scale.contiguous()
        s13 = gemm1_weights_scale.contiguous()
        s2 = gemm2_weights_scale.contiguous()
        code = load_library().moe_b200_run_noalloc(
            logits.data_ptr(), bias.data_ptr(), bias_dtype, hidden_states.data_ptr(), hs_scale.data_ptr(),
            gemm1_weights.data_ptr(), s13.data_ptr(), gemm2_weights.data_ptr(), s2.data_ptr(),
            int(local_expert_offset), float(routed_scaling_factor), T, output.data_ptr(),
            torch.cuda.current_stream(dev).cuda_stream)
    _raise_on(code, "moe_b200_run_noalloc")
    return output


def noalloc_read_status(device: torch.device | None = None) -> int:
    """Status word of the last moe_b200_run_noalloc on ``device`` (0 = clean)."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    st = ctypes.c_uint32(0)
    with torch.cuda.device(dev):
        code = load_library().moe_b200_noalloc_read_status(ctypes.byref(st),
                                                            torch.cuda.current_stream(dev).cuda_stream)
    if code not in (0, 7):
        _raise_on(code, "moe_b200_noalloc_read_status")
    return int(st.value)


def run(routing_logits, routing_bias, hidden_states, hidden_states_scale, gemm1_weights,
        gemm1_weights_scale, gemm2_weights, gemm2_weights_scale, local_expert_offset,
        routed_scaling_factor) -> torch.Tensor:
    """Value-returning form of the reference entry point (solution/cuda/main.py:31-54)."""
    T = _check_inputs(routing_logits, routing_bias, hidden_states, hidden_states_scale,
                      gemm1_weights, gemm1_weights_scale, gemm2_weights, gemm2_weights_scale)
    out = torch.empty((T, H), dtype=torch.bfloat16, device=routing_logits.device)
    return run_dps(routing_logits, routing_bias, hidden_states, hidden_states_scale, gemm1_weights,
                   gemm1_weights_scale, gemm2_weights, gemm2_weights_scale, local_expert_offset,
                   routed_scaling_factor, out)


def route(routing_logits, routing_bias, routed_scaling_factor) -> tuple[torch.Tensor, torch.Tensor]:
    """Routing only: (topk_idx int32 [T, 8] best first, topk_w fp32 [T, 8])."""
    _check(routing_logits.is_cuda and routing_logits.dtype == torch.float32
           and routing_logits.dim() == 2 and routing_logits.size(1) == E_GLOBAL,
           f"routing_logits must be a CUDA float32 [T, {E_GLOBAL}] tensor")
    T = routing_logits.size(0)
    dev = routing_logits.device
    idx = torch.empty((T, TOP_K), dtype=torch.int32, device=dev)
    w = torch.empty((T, TOP_K), dtype=torch.float32, device=dev)
    if T == 0:
        return idx, w
    lib = load_library()
    with torch.cuda.device(dev):
        logits = routing_logits.contiguous()
        bias, bias_dtype = _bias_arg(routing_bias.to(dev))
        code = lib.moe_b200_route(logits.data_ptr(), bias.data_ptr(), bias_dtype, T,
                                  float(routed_scaling_factor), idx.data_ptr(), w.data_ptr(),
                                  torch.cuda.current_stream(dev).cuda_stream)
    _raise_on(code, "moe_b200_route")
    return idx, w


def read_status(workspace: torch.Tensor) -> int:
    """Device status word of the last call that used ``workspace`` (0 = clean)."""
    lib = load_library()
    st = ctypes.c_uint32(0)
    with torch.cuda.device(workspace.device):
        lib.moe_b200_read_status(workspace.data_ptr(), ctypes.byref(st),
                                 torch.cuda.current_stream(workspace.device).cuda_stream)
    return int(st.value)


NUM_STAGE_EVENTS = 7
STAGE_NAMES = ("clear", "route", "permute", "gemm1", "gemm2", "finalize")


def set_stage_events(events) -> None:
    """Profiling hook: record these 7 torch.cuda.Event objects at the stage
    boundaries of every later run on this thread (None switches it off).
    Each event must already have been recorded once (torch creates the
    underlying CUDA event lazily)."""
    lib = load_library()
    if events is None:
        _raise_on(lib.moe_b200_set_stage_events(None, 0), "moe_b200_set_stage_events")
        return
    arr = (ctypes.c_void_p * NUM_STAGE_EVENTS)(*[ctypes.c_void_p(e.cuda_event) for e in events])
    _raise_on(lib.moe_b200_set_stage_events(arr, NUM_STAGE_EVENTS), "moe_b200_set_stage_events")
