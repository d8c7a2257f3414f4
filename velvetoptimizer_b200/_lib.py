"""ctypes binding of ``libvesper_moe.so`` (the C ABI declared in include/vesper_moe.h).

The library is the only compute path: if it is missing, importing the op raises instead
of falling back to anything else.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, c_char_p, c_float, c_int, c_int32, c_int64, c_size_t, c_void_p

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "lib", "libvesper_moe.so")

VMOE_OK = 0
VMOE_ERR_INVALID_ARG = 1
VMOE_ERR_UNSUPPORTED_SHAPE = 2
VMOE_ERR_CUDA = 3
VMOE_ERR_NCCL = 4
VMOE_ERR_TIMEOUT = 5
VMOE_ERR_DEVICE_STATUS = 6
VMOE_ERR_NOT_READY = 7
VMOE_ERR_WORKSPACE = 8

VMOE_F32 = 0
VMOE_BF16 = 1

# size of the static scratch array behind vmoe_forward_no_alloc
VMOE_NO_ALLOC_WORKSPACE_BYTES = 64 << 20

# every symbol include/vesper_moe.h declares
EXPORTED = (
    "vmoe_create", "vmoe_destroy", "vmoe_set_weights", "vmoe_workspace_size",
    "vmoe_workspace_layout", "vmoe_forward", "vmoe_forward_no_alloc",
    "vmoe_device_status", "vmoe_set_profiling", "vmoe_stage_times", "vmoe_stage_name",
    "vmoe_last_launch_count", "vmoe_last_error", "vmoe_status_string", "vmoe_abi_version",
    "vmoe_create_ep", "vmoe_ep_workspace_size", "vmoe_ep_route", "vmoe_ep_experts",
    "vmoe_ep_combine", "vmoe_ep_p2p_setup", "vmoe_ep_p2p_connect", "vmoe_ep_p2p_workspace_size",
    "vmoe_ep_p2p_forward", "vmoe_ep_p2p_host_workspace_size", "vmoe_ep_p2p_forward_host",
    "vmoe_gemm_tile_rows", "vmoe_segment_align", "vmoe_ffn_create",
    "vmoe_ffn_workspace_size",
    "vmoe_ffn_forward", "vmoe_forward_host_workspace_size", "vmoe_forward_host",
    "vmoe_set_norm", "vmoe_forward_residual", "vmoe_set_training", "vmoe_train_workspace_size",
    "vmoe_forward_train", "vmoe_backward", "vmoe_backward_stage_times",
    "vmoe_backward_stage_name",
)


class VmoeGrads(ctypes.Structure):
    """vmoe_grads: fp32 device pointers of the parameter gradients."""
    _fields_ = [(n, c_void_p) for n in ("router_w", "router_b", "gate_w", "gate_b", "up_w", "up_b",
                                         "down_w", "down_b")]


class VmoeConfig(ctypes.Structure):
    _fields_ = [
        ("hidden", c_int64),
        ("inter", c_int64),
        ("num_experts", c_int32),
        ("top_k", c_int32),
        ("lora_rank", c_int32),
        ("lora_scaling", c_float),
        ("era_gamma", c_float),
        ("dtype", c_int32),
        ("capacity", c_int64),
    ]


class VmoeWeights(ctypes.Structure):
    _fields_ = [(n, c_void_p) for n in (
        "router_w", "router_b", "gate_w", "gate_b", "up_w", "up_b", "down_w", "down_b",
        "gate_lora_down_w", "gate_lora_down_b", "gate_lora_up_w", "gate_lora_up_b",
        "up_lora_down_w", "up_lora_down_b", "up_lora_up_w", "up_lora_up_b",
    )]


class VmoeWsLayout(ctypes.Structure):
    _fields_ = [("slot_of", c_size_t), ("expert_offsets", c_size_t), ("num_tiles", c_size_t),
                ("x_perm", c_size_t), ("h", c_size_t), ("y", c_size_t), ("max_rows", c_int64),
                ("h_ld", c_int64), ("y_ld", c_int64), ("total", c_size_t)]


class VmoeError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(msg)
        self.code = code


_lib = None


def load() -> ctypes.CDLL:
    """Load the library once; raise if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `python -m velvetoptimizer_b200.build` "
            "(there is no non-CUDA fallback)")
    lib = ctypes.CDLL(LIB_PATH)
    H = c_void_p
    lib.vmoe_create.argtypes = [POINTER(VmoeConfig), c_int, POINTER(H)]
    lib.vmoe_create.restype = c_int
    lib.vmoe_destroy.argtypes = [H]
    lib.vmoe_destroy.restype = c_int
    lib.vmoe_set_weights.argtypes = [H, POINTER(VmoeWeights), c_void_p]
    lib.vmoe_set_weights.restype = c_int
    lib.vmoe_workspace_size.argtypes = [H, c_int64, POINTER(c_size_t)]
    lib.vmoe_workspace_size.restype = c_int
    lib.vmoe_workspace_layout.argtypes = [H, c_int64, POINTER(VmoeWsLayout)]
    lib.vmoe_workspace_layout.restype = c_int
    lib.vmoe_forward.argtypes = [H, c_void_p, c_int64, c_void_p, c_void_p, c_void_p, c_void_p,
                                 c_void_p, c_void_p, c_void_p, c_size_t, c_void_p]
    lib.vmoe_forward.restype = c_int
    lib.vmoe_forward_no_alloc.argtypes = [H, c_void_p, c_int64, c_void_p, c_void_p, c_void_p,
                                          c_void_p, c_void_p, c_void_p, c_void_p]
    lib.vmoe_forward_no_alloc.restype = c_int
    lib.vmoe_forward_host_workspace_size.argtypes = [H, c_int64, c_int, POINTER(c_size_t)]
    lib.vmoe_forward_host_workspace_size.restype = c_int
    lib.vmoe_forward_host.argtypes = [H, c_void_p, c_int64, c_void_p, c_void_p, c_int, c_void_p,
                                      c_size_t, c_void_p]
    lib.vmoe_forward_host.restype = c_int
    lib.vmoe_backward_stage_times.argtypes = [H, POINTER(c_float), c_int, POINTER(c_int),
                                              POINTER(c_int)]
    lib.vmoe_backward_stage_times.restype = c_int
    lib.vmoe_backward_stage_name.argtypes = [c_int]
    lib.vmoe_backward_stage_name.restype = c_char_p
    lib.vmoe_set_training.argtypes = [H, c_int, c_void_p]
    lib.vmoe_set_training.restype = c_int
    lib.vmoe_train_workspace_size.argtypes = [H, c_int64, POINTER(c_size_t), POINTER(c_size_t)]
    lib.vmoe_train_workspace_size.restype = c_int
    lib.vmoe_forward_train.argtypes = [H, c_void_p, c_int64, c_void_p, c_void_p, c_void_p,
                                       c_void_p, c_size_t, c_void_p]
    lib.vmoe_forward_train.restype = c_int
    lib.vmoe_backward.argtypes = [H, c_void_p, c_void_p, c_int64, c_void_p, c_void_p,
                                  POINTER(VmoeGrads), c_void_p, c_size_t, c_void_p, c_size_t,
                                  c_void_p]
    lib.vmoe_backward.restype = c_int
    lib.vmoe_set_norm.argtypes = [H, c_void_p, c_void_p, c_float, c_void_p]
    lib.vmoe_set_norm.restype = c_int
    lib.vmoe_forward_residual.argtypes = lib.vmoe_forward.argtypes
    lib.vmoe_forward_residual.restype = c_int
    lib.vmoe_create_ep.argtypes = [POINTER(VmoeConfig), c_int, c_int, c_int, POINTER(H)]
    lib.vmoe_create_ep.restype = c_int
    lib.vmoe_ep_workspace_size.argtypes = [H, c_int64, c_int64, POINTER(c_size_t)]
    lib.vmoe_ep_workspace_size.restype = c_int
    lib.vmoe_ep_route.argtypes = [H, c_void_p, c_int64, c_void_p, c_void_p, c_void_p, c_void_p,
                                  c_void_p, c_size_t, c_void_p]
    lib.vmoe_ep_route.restype = c_int
    lib.vmoe_ep_experts.argtypes = [H, c_void_p, c_int64, c_void_p, c_void_p, c_void_p,
                                    c_void_p, c_size_t, c_void_p]
    lib.vmoe_ep_experts.restype = c_int
    lib.vmoe_ep_combine.argtypes = [H, c_void_p, c_int64, c_void_p, c_void_p, c_size_t, c_void_p]
    lib.vmoe_ep_combine.restype = c_int
    lib.vmoe_ep_p2p_setup.argtypes = [H, c_int64, c_int, c_void_p]
    lib.vmoe_ep_p2p_setup.restype = c_int
    lib.vmoe_ep_p2p_connect.argtypes = [H, c_void_p]
    lib.vmoe_ep_p2p_connect.restype = c_int
    lib.vmoe_ep_p2p_workspace_size.argtypes = [H, c_int64, POINTER(c_size_t)]
    lib.vmoe_ep_p2p_workspace_size.restype = c_int
    lib.vmoe_ep_p2p_forward.argtypes = [H, c_void_p, c_int64, c_void_p, c_void_p, c_void_p,
                                        c_void_p, c_size_t, c_void_p]
    lib.vmoe_ep_p2p_forward.restype = c_int
    lib.vmoe_ep_p2p_host_workspace_size.argtypes = [H, POINTER(c_size_t)]
    lib.vmoe_ep_p2p_host_workspace_size.restype = c_int
    lib.vmoe_ep_p2p_forward_host.argtypes = [H, c_void_p, c_int64, c_void_p, c_void_p, c_void_p,
                                             c_size_t, c_void_p]
    lib.vmoe_ep_p2p_forward_host.restype = c_int
    lib.vmoe_device_status.argtypes = [H, POINTER(c_int32), c_void_p]
    lib.vmoe_device_status.restype = c_int
    lib.vmoe_set_profiling.argtypes = [H, c_int]
    lib.vmoe_set_profiling.restype = c_int
    lib.vmoe_stage_times.argtypes = [H, POINTER(c_float), c_int, POINTER(c_int), POINTER(c_int)]
    lib.vmoe_stage_times.restype = c_int
    lib.vmoe_stage_name.argtypes = [c_int]
    lib.vmoe_stage_name.restype = c_char_p
    lib.vmoe_last_launch_count.argtypes = [H]
    lib.vmoe_last_launch_count.restype = c_int
    lib.vmoe_ffn_create.argtypes = [POINTER(VmoeConfig), c_int, POINTER(H)]
    lib.vmoe_ffn_create.restype = c_int
    lib.vmoe_ffn_workspace_size.argtypes = [H, c_int64, POINTER(c_size_t)]
    lib.vmoe_ffn_workspace_size.restype = c_int
    lib.vmoe_ffn_forward.argtypes = [H, c_void_p, c_int64, c_void_p, c_void_p, c_size_t, c_void_p]
    lib.vmoe_ffn_forward.restype = c_int
    lib.vmoe_gemm_tile_rows.argtypes = [H]
    lib.vmoe_gemm_tile_rows.restype = c_int
    lib.vmoe_segment_align.argtypes = [H, c_int64]
    lib.vmoe_segment_align.restype = c_int
    lib.vmoe_last_error.argtypes = [H]
    lib.vmoe_last_error.restype = c_char_p
    lib.vmoe_status_string.argtypes = [c_int]
    lib.vmoe_status_string.restype = c_char_p
    lib.vmoe_abi_version.argtypes = []
    lib.vmoe_abi_version.restype = c_int
    _lib = lib
    return lib


def check(rc: int, handle=None, what: str = "vmoe call") -> None:
    """Raise VmoeError for a non-zero status, with the handle's error text."""
    if rc == VMOE_OK:
        return
    lib = load()
    detail = ""
    if handle:
        detail = (lib.vmoe_last_error(handle) or b"").decode()
    status = (lib.vmoe_status_string(rc) or b"").decode()
    raise VmoeError(rc, f"{what} failed: {status}" + (f" ({detail})" if detail else ""))


class Handle:
    """Owns one ``vmoe_handle`` (one layer configuration on one device)."""

    def __init__(self, cfg: VmoeConfig, device: int, dense: bool = False):
        self.lib = load()
        self.cfg = cfg
        self.device = device
        self.ptr = c_void_p()
        create = self.lib.vmoe_ffn_create if dense else self.lib.vmoe_create
        check(create(ctypes.byref(cfg), device, ctypes.byref(self.ptr)), None,
              "vmoe_ffn_create" if dense else "vmoe_create")

    def close(self) -> None:
        if self.ptr:
            self.lib.vmoe_destroy(self.ptr)
            self.ptr = c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def workspace_size(self, tokens: int) -> int:
        n = c_size_t()
        check(self.lib.vmoe_workspace_size(self.ptr, tokens, ctypes.byref(n)), self.ptr,
              "vmoe_workspace_size")
        return n.value

    def workspace_layout(self, tokens: int) -> VmoeWsLayout:
        lay = VmoeWsLayout()
        check(self.lib.vmoe_workspace_layout(self.ptr, tokens, ctypes.byref(lay)), self.ptr,
              "vmoe_workspace_layout")
        return lay

    def set_weights(self, w: VmoeWeights, stream: int) -> None:
        check(self.lib.vmoe_set_weights(self.ptr, ctypes.byref(w), c_void_p(stream)), self.ptr,
              "vmoe_set_weights")

    def forward(self, x, tokens, out, logits, idx, topw, counts, aux, ws, ws_bytes, stream):
        rc = self.lib.vmoe_forward(self.ptr, x, tokens, out, logits, idx, topw, counts, aux, ws,
                                   ws_bytes, c_void_p(stream))
        check(rc, self.ptr, "vmoe_forward")

    def set_training(self, enable: bool, stream: int) -> None:
        check(self.lib.vmoe_set_training(self.ptr, 1 if enable else 0, c_void_p(stream)), self.ptr,
              "vmoe_set_training")

    def train_workspace_size(self, tokens: int) -> tuple[int, int]:
        a, b = c_size_t(), c_size_t()
        check(self.lib.vmoe_train_workspace_size(self.ptr, tokens, ctypes.byref(a), ctypes.byref(b)),
              self.ptr, "vmoe_train_workspace_size")
        return a.value, b.value

    def forward_train(self, x, tokens, out, logits, aux, saved, saved_bytes, stream):
        check(self.lib.vmoe_forward_train(self.ptr, x, tokens, out, logits, aux, saved,
                                          saved_bytes, c_void_p(stream)), self.ptr,
              "vmoe_forward_train")

    def backward(self, x, dout, tokens, daux, dx, grads: "VmoeGrads", saved, saved_bytes, scratch,
                 scratch_bytes, stream):
        check(self.lib.vmoe_backward(self.ptr, x, dout, tokens, daux, dx, ctypes.byref(grads),
                                     saved, saved_bytes, scratch, scratch_bytes, c_void_p(stream)),
              self.ptr, "vmoe_backward")

    def set_norm(self, weight, bias, eps: float, stream: int) -> None:
        """LayerNorm parameters (device pointers or None) of the fused pre-norm block."""
        check(self.lib.vmoe_set_norm(self.ptr, weight, bias, float(eps), c_void_p(stream)),
              self.ptr, "vmoe_set_norm")

    def forward_residual(self, x, tokens, out, logits, idx, topw, counts, aux, ws, ws_bytes,
                         stream):
        rc = self.lib.vmoe_forward_residual(self.ptr, x, tokens, out, logits, idx, topw, counts,
                                            aux, ws, ws_bytes, c_void_p(stream))
        check(rc, self.ptr, "vmoe_forward_residual")

    def host_workspace_size(self, tokens: int, chunks: int = 0) -> int:
        n = c_size_t()
        check(self.lib.vmoe_forward_host_workspace_size(self.ptr, tokens, chunks, ctypes.byref(n)),
              self.ptr, "vmoe_forward_host_workspace_size")
        return n.value

    def forward_host(self, x_host, tokens, out_host, aux_host, chunks, ws, ws_bytes, stream):
        rc = self.lib.vmoe_forward_host(self.ptr, x_host, tokens, out_host, aux_host, chunks, ws,
                                        ws_bytes, c_void_p(stream))
        check(rc, self.ptr, "vmoe_forward_host")

    def device_status(self, stream: int) -> int:
        code = c_int32()
        check(self.lib.vmoe_device_status(self.ptr, ctypes.byref(code), c_void_p(stream)),
              self.ptr, "vmoe_device_status")
        return code.value

    def set_profiling(self, forwards: int) -> None:
        """Record per-stage events for the next ``forwards`` forwards (0 = off)."""
        check(self.lib.vmoe_set_profiling(self.ptr, int(forwards)), self.ptr, "vmoe_set_profiling")

    def stage_times(self) -> tuple[dict[str, float], int]:
        """(average ms per stage, number of forwards averaged); restarts recording."""
        buf = (c_float * 16)()
        n, f = c_int(), c_int()
        check(self.lib.vmoe_stage_times(self.ptr, buf, 16, ctypes.byref(n), ctypes.byref(f)),
              self.ptr, "vmoe_stage_times")
        return {self.lib.vmoe_stage_name(i).decode(): float(buf[i]) for i in range(n.value)}, f.value

    def backward_stage_times(self) -> tuple[dict[str, float], int]:
        """(average ms per backward stage, number of backwards averaged); restarts recording."""
        buf = (c_float * 16)()
        n, f = c_int(), c_int()
        check(self.lib.vmoe_backward_stage_times(self.ptr, buf, 16, ctypes.byref(n), ctypes.byref(f)),
              self.ptr, "vmoe_backward_stage_times")
        return ({self.lib.vmoe_backward_stage_name(i).decode(): float(buf[i]) for i in range(n.value)},
                f.value)

    def last_launch_count(self) -> int:
        return int(self.lib.vmoe_last_launch_count(self.ptr))
