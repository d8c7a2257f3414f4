"""Drive the C ABI directly from numpy inputs (used by the GPU parity tests and smoke()).

Everything crosses the boundary as raw device pointers in the same layout the reference's
parameters have ([E, out, in] stacks), exactly as a non-Python caller would bind it.
"""
from __future__ import annotations

import ctypes

import numpy as np
import torch

from velvetoptimizer_b200 import _lib

_WEIGHT_KEYS = {
    "router_w": "w_r", "router_b": "b_r",
    "gate_w": "w_g", "gate_b": "b_g", "up_w": "w_u", "up_b": "b_u",
    "down_w": "w_d", "down_b": "b_d",
    "gate_lora_down_w": "a_g", "gate_lora_down_b": "ba_g",
    "gate_lora_up_w": "l_g", "gate_lora_up_b": "bl_g",
    "up_lora_down_w": "a_u", "up_lora_down_b": "ba_u",
    "up_lora_up_w": "l_u", "up_lora_up_b": "bl_u",
}


def abi_config(case, dtype: str, capacity: int = 0) -> _lib.VmoeConfig:
    return _lib.VmoeConfig(hidden=case.hidden, inter=case.inter, num_experts=case.experts,
                           top_k=case.top_k, lora_rank=case.lora_rank,
                           lora_scaling=case.lora_scaling, era_gamma=case.era_gamma,
                           dtype=_lib.VMOE_F32 if dtype == "f32" else _lib.VMOE_BF16,
                           capacity=capacity)


class AbiLayer:
    """One handle + uploaded weights for a case; ``run(x)`` returns numpy results."""

    def __init__(self, case, inputs: dict, dtype: str = "f32", device: int = 0,
                 capacity: int = 0):
        self.case, self.dtype, self.device = case, dtype, device
        self.tdtype = torch.float32 if dtype == "f32" else torch.bfloat16
        self.handle = _lib.Handle(abi_config(case, dtype, capacity), device)
        dev = torch.device("cuda", device)
        w = {k: torch.from_numpy(np.ascontiguousarray(inputs[v])).to(dev, self.tdtype)
             for k, v in _WEIGHT_KEYS.items()}
        vw = _lib.VmoeWeights(**{k: ctypes.c_void_p(t.data_ptr()) for k, t in w.items()})
        self.stream = torch.cuda.current_stream(dev)
        self.handle.set_weights(vw, self.stream.cuda_stream)
        self.stream.synchronize()
        del w
        self.ws = None

    def run(self, x_np: np.ndarray, *, profile: bool = False) -> dict:
        c = self.case
        dev = torch.device("cuda", self.device)
        T = x_np.shape[0]
        x = torch.from_numpy(np.ascontiguousarray(x_np)).to(dev, self.tdtype)
        res = self.run_device(x, profile=profile)
        out = {k: v.float().cpu().numpy() if v.dtype != torch.int32 else v.cpu().numpy()
               for k, v in res.items()}
        out["aux"] = out["aux"].reshape(())
        out["topk_idx"] = out["topk_idx"].astype(np.int64)
        assert out["out"].shape == (T, c.hidden)
        return out

    def run_device(self, x: torch.Tensor, *, profile: bool = False) -> dict:
        c = self.case
        dev = x.device
        T = x.shape[0]
        need = self.handle.workspace_size(T)
        if self.ws is None or self.ws.numel() < need:
            self.ws = torch.empty(max(need, 256), dtype=torch.uint8, device=dev)
        r = {
            "out": torch.empty((T, c.hidden), dtype=self.tdtype, device=dev),
            "logits": torch.empty((T, c.experts), dtype=torch.float32, device=dev),
            "topk_idx": torch.empty((T, c.top_k), dtype=torch.int32, device=dev),
            "topk_w": torch.empty((T, c.top_k), dtype=torch.float32, device=dev),
            "counts": torch.empty((c.experts,), dtype=torch.int32, device=dev),
            "aux": torch.empty((1,), dtype=torch.float32, device=dev),
        }
        if profile:
            self.handle.set_profiling(1)
        self.handle.forward(x.data_ptr(), T, r["out"].data_ptr(), r["logits"].data_ptr(),
                            r["topk_idx"].data_ptr(), r["topk_w"].data_ptr(),
                            r["counts"].data_ptr(), r["aux"].data_ptr(), self.ws.data_ptr(),
                            self.ws.numel(), self.stream.cuda_stream)
        self.stream.synchronize()
        status = self.handle.device_status(self.stream.cuda_stream)
        assert status == 0, f"device status 0x{status:x}"
        return r

    def close(self):
        self.handle.close()
