"""The allocation-free forward (vmoe_forward_no_alloc) against the regular vmoe_forward.

vmoe_forward_no_alloc serves callers that cannot allocate device memory while they run
the layer (a serving thread under a fixed memory budget, a real-time loop, an engine with
no caching allocator): it takes its scratch from a static 64 MiB device array instead of
a caller workspace.  These tests call both entry points through the C ABI on the same
inputs, twice in a row for the static one (the array keeps the previous call's contents),
after first filling the array with an unrelated, larger layer's scratch, and require the
results to be bit-identical: both entry points run the same kernels on the same inputs,
and no scratch is read before the call has written it.  The file is named to be collected
last.
"""
import ctypes

import numpy as np
import pytest
import torch

from oracle import moe_oracle as O
from oracle.inputs import MoECase, bf16_inputs, make_inputs
from tests.abi_runner import AbiLayer
from velvetoptimizer_b200 import _lib

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _need_cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")


def _no_alloc_call(layer, x):
    """Run vmoe_forward_no_alloc; returns numpy results (caller-owned outputs only)."""
    c = layer.case
    dev = x.device
    T = x.shape[0]
    out = torch.empty((T, c.hidden), dtype=x.dtype, device=dev)
    idx = torch.empty((T, c.top_k), dtype=torch.int32, device=dev)
    counts = torch.empty((c.experts,), dtype=torch.int32, device=dev)
    aux = torch.empty((1,), dtype=torch.float32, device=dev)
    rc = _lib.load().vmoe_forward_no_alloc(layer.handle.ptr, ctypes.c_void_p(x.data_ptr()), T,
                                           ctypes.c_void_p(out.data_ptr()), None,
                                           ctypes.c_void_p(idx.data_ptr()), None,
                                           ctypes.c_void_p(counts.data_ptr()),
                                           ctypes.c_void_p(aux.data_ptr()),
                                           ctypes.c_void_p(layer.stream.cuda_stream))
    _lib.check(rc, layer.handle.ptr, "vmoe_forward_no_alloc")
    layer.stream.synchronize()
    assert layer.handle.device_status(layer.stream.cuda_stream) == 0
    return {"out": out.float().cpu().numpy(), "topk_idx": idx.cpu().numpy().astype(np.int64),
            "counts": counts.cpu().numpy(), "aux": float(aux.item())}


def _dirty_the_array(dtype):
    """Fill the static array with another layer's scratch: more tokens, more experts, a
    larger top-K and other widths, so stale slots, offsets and rows sit everywhere."""
    other = MoECase(tokens=200, hidden=768, inter=1536, experts=16, top_k=4, bias_std=0.05,
                    seed=33)
    oinp = make_inputs(other)
    if dtype == "bf16":
        oinp = bf16_inputs(oinp)
    olayer = AbiLayer(other, oinp, dtype)
    assert olayer.handle.workspace_size(other.tokens) <= _lib.VMOE_NO_ALLOC_WORKSPACE_BYTES
    x = torch.from_numpy(oinp["x"]).cuda().to(olayer.tdtype)
    _no_alloc_call(olayer, x)
    olayer.close()


@pytest.mark.parametrize("dtype,tol", [("bf16", 2e-2), ("f32", 1e-5)])
def test_no_alloc_matches_forward_twice(dtype, tol):
    # a decode-shaped batch: few tokens, so the scratch fits the static array
    case = MoECase(tokens=64, hidden=512, inter=1024, experts=8, top_k=2, bias_std=0.02, seed=31)
    inp = make_inputs(case)
    if dtype == "bf16":
        inp = bf16_inputs(inp)
    layer = AbiLayer(case, inp, dtype)
    assert layer.handle.workspace_size(case.tokens) <= _lib.VMOE_NO_ALLOC_WORKSPACE_BYTES
    ref = layer.run(inp["x"])                      # vmoe_forward, caller workspace
    x = torch.from_numpy(inp["x"]).cuda().to(layer.tdtype)
    _dirty_the_array(dtype)
    for _ in range(2):                             # two calls in a row share the array
        got = _no_alloc_call(layer, x)
        # the same kernels on the same inputs: bit-identical (tol bounds the oracle gap)
        assert np.array_equal(got["out"], ref["out"])
        assert np.array_equal(got["topk_idx"], ref["topk_idx"])
        assert np.array_equal(got["counts"], ref["counts"])
        assert got["aux"] == float(ref["aux"])
    oracle = O.moe_forward(inp, case, force_idx=got["topk_idx"])
    assert O.norm_rel_err(got["out"], oracle["out"]) < tol
    # a smaller batch after the larger one: the array still holds the 64-token call's rows
    ref9 = layer.run(inp["x"][:9])
    got9 = _no_alloc_call(layer, x[:9].contiguous())
    assert np.array_equal(got9["out"], ref9["out"])
    layer.close()


def test_no_alloc_reports_negative_token_counts():
    case = MoECase(tokens=8, hidden=128, inter=256, experts=4, top_k=2, seed=34)
    layer = AbiLayer(case, bf16_inputs(make_inputs(case)), "bf16")
    x = torch.zeros((8, case.hidden), dtype=torch.bfloat16, device="cuda")  # never read
    rc = _lib.load().vmoe_forward_no_alloc(layer.handle.ptr, ctypes.c_void_p(x.data_ptr()), -3,
                                           ctypes.c_void_p(x.data_ptr()), None, None, None,
                                           None, None, ctypes.c_void_p(layer.stream.cuda_stream))
    assert rc == _lib.VMOE_ERR_INVALID_ARG
    assert "tokens must be >= 0" in _lib.load().vmoe_last_error(layer.handle.ptr).decode()
    layer.close()


def test_no_alloc_rejects_batches_beyond_the_static_array():
    case = MoECase(tokens=64, hidden=512, inter=1024, experts=8, top_k=2, seed=32)
    layer = AbiLayer(case, bf16_inputs(make_inputs(case)), "bf16")
    big = 200_000
    assert layer.handle.workspace_size(big) > _lib.VMOE_NO_ALLOC_WORKSPACE_BYTES
    x = torch.zeros((8, case.hidden), dtype=torch.bfloat16, device="cuda")  # never read
    rc = _lib.load().vmoe_forward_no_alloc(layer.handle.ptr, ctypes.c_void_p(x.data_ptr()), big,
                                           ctypes.c_void_p(x.data_ptr()), None, None, None,
                                           None, None, ctypes.c_void_p(layer.stream.cuda_stream))
    assert rc == _lib.VMOE_ERR_WORKSPACE
    msg = _lib.load().vmoe_last_error(layer.handle.ptr).decode()
    assert "static workspace holds" in msg and "64 MiB" in msg
    layer.close()
