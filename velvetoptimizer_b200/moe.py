"""Drop-in MoE layer for VelvetOptimizer's ``MoELayer`` (python/vesper/model.py:305-385).

``MoELayer(config)`` has the reference's submodule names, so its ``state_dict`` keys are
the reference's (``router.*``, ``experts.{e}.{gate_proj,up_proj}.{base,lora_down,lora_up}.*``,
``experts.{e}.{gate_proj,up_proj}.proj_a``, ``experts.{e}.down_proj.*``) and a reference
checkpoint loads unchanged.  ``forward(x[B,S,H]) -> (out[B,S,H], aux_loss[])`` keeps the
reference's return signature so ``TransformerLayer`` (model.py:419-420) does not change;
``return_router_logits=True`` also returns the router logits.

The forward calls the C ABI (include/vesper_moe.h) on torch's current stream, through
the custom op ``torch.ops.vesper_moe.forward`` under a tracer (torch.compile, export) and
through the op's body directly in eager mode.  There is no CPU fallback: CPU tensors, a
missing library or an unsupported dtype raise.

Training (the reference trains through this layer, python/train.py:465): with gradients
wanted on a bf16 input, the forward runs ``vmoe_forward_train`` inside an autograd
Function whose backward is ``vmoe_backward`` (dx, the router's and every expert's weight
and bias gradients); the FlyLoRA factors' gradients follow from the effective-weight
gradients by the chain rule of W + s U D (model.py:123-126).  fp32 inputs have no
backward here: they run the forward only (with a warning when gradients were wanted).
"""
from __future__ import annotations

import ctypes
import itertools
import math
import warnings
import weakref

import torch
import torch.nn as nn
from torch.optim.optimizer import register_optimizer_step_post_hook

from . import _lib
from .config import MoEConfig

try:  # the (data pointer, version) pairs of a parameter list in one native call
    from .lib._param_key import pairs as _native_pairs
except ImportError:  # not built: the same pairs read one parameter at a time
    _native_pairs = None

_DTYPES = {torch.float32: _lib.VMOE_F32, torch.bfloat16: _lib.VMOE_BF16}

# Every forward checks that the packed weights are current.  Walking the module tree for
# its parameters costs about a millisecond with 64 experts (900 parameters), more than a
# decode-sized forward on the GPU, so the layers keep their parameter list and rebuild it
# only after a parameter or submodule has been (re)assigned on one of their own modules
# (_STRUCTURE_GEN, bumped by torch's registration hooks for the modules in _OWNED).
# The weight key holds each parameter's data pointer and version (load_state_dict and
# in-place updates through the parameter bump the version, `.data` assignment moves the
# pointer) plus two generations for writes that change neither:
#   * _WRITE_GEN, bumped after every torch optimizer step: optimizers commonly write
#     through `p.data` (VelvetOptimizer does, python/vesper/optimizer.py:176,212), which
#     leaves the parameter's version untouched;
#   * the layer's own counter, bumped by ``mark_weights_dirty()`` for any other such write.
# The hooks are installed when the first layer is built, not at import.
_STRUCTURE_GEN = [0]
_WRITE_GEN = [0]
_OWNED: "weakref.WeakSet[nn.Module]" = weakref.WeakSet()
_HOOKS: list = []


def _structure_changed(module, _name, _obj):
    if module in _OWNED:
        _STRUCTURE_GEN[0] += 1
    return None  # keep the registered object


def _optimizer_stepped(_optimizer, _args, _kwargs):
    _WRITE_GEN[0] += 1


def _install_hooks() -> None:
    if _HOOKS:
        return
    _HOOKS.append(nn.modules.module.register_module_parameter_registration_hook(_structure_changed))
    _HOOKS.append(nn.modules.module.register_module_module_registration_hook(_structure_changed))
    _HOOKS.append(register_optimizer_step_post_hook(_optimizer_stepped))


class FlyLoRALinear(nn.Module):
    """Parameter container with the reference FlyLoRALinear's names (model.py:83-121).

    ``base`` [out,in], ``lora_down`` [r,in], ``lora_up`` [out,r] (zero-initialised, so the
    branch starts switched off, model.py:120) and the unused ``proj_a`` buffer [in,r]
    (model.py:107-113).  Its math runs inside the fused op, folded into ``base``.
    """

    def __init__(self, in_features: int, out_features: int, rank: int = 16,
                 alpha: float = 32.0, sparsity: float = 0.25):
        super().__init__()
        self.in_features, self.out_features, self.rank = in_features, out_features, rank
        self.scaling = alpha / rank
        self.base = nn.Linear(in_features, out_features)
        proj = torch.randn(in_features, rank)
        proj = proj * (torch.rand_like(proj) > sparsity).float()
        self.register_buffer("proj_a", proj / proj.norm(dim=0, keepdim=True).clamp(min=1e-8))
        self.lora_down = nn.Linear(in_features, rank, bias=True)
        self.lora_up = nn.Linear(rank, out_features, bias=True)
        nn.init.kaiming_uniform_(self.lora_down.weight, a=math.sqrt(5))
        nn.init.zeros_(self.lora_up.weight)

    def forward(self, x):  # pragma: no cover - the fused op is the only compute path
        raise RuntimeError("FlyLoRALinear is evaluated inside the fused MoE op")


class ExpertFFN(nn.Module):
    """Parameter container with the reference ExpertFFN's names (model.py:277-293)."""

    def __init__(self, cfg: MoEConfig):
        super().__init__()
        args = (cfg.hidden_size, cfg.intermediate_size, cfg.flylora_rank, cfg.flylora_alpha,
                cfg.flylora_sparsity)
        self.gate_proj = FlyLoRALinear(*args)
        self.up_proj = FlyLoRALinear(*args)
        self.down_proj = nn.Linear(cfg.intermediate_size, cfg.hidden_size)

    def forward(self, x):  # pragma: no cover
        raise RuntimeError("ExpertFFN is evaluated inside the fused MoE op")


# ---------------------------------------------------------------------------------------
# handle registry + custom op
# ---------------------------------------------------------------------------------------
_HANDLES: dict[int, "_Packed"] = {}
_ids = itertools.count(1)


class _Packed:
    """A C-ABI handle with packed weights plus a growable workspace."""

    def __init__(self, handle: _lib.Handle, key):
        self.handle = handle
        self.key = key
        self.ws: torch.Tensor | None = None
        self.id = next(_ids)
        _HANDLES[self.id] = self

    def workspace(self, tokens: int, device) -> torch.Tensor:
        return self.scratch(self.handle.workspace_size(tokens), device)

    def scratch(self, need: int, device) -> torch.Tensor:
        if self.ws is None or self.ws.numel() < need:
            self.ws = torch.empty(max(need, 256), dtype=torch.uint8, device=device)
        return self.ws

    def release(self):
        _HANDLES.pop(self.id, None)
        self.handle.close()


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _moe_forward(x: torch.Tensor, handle_id: int, want_logits: bool) -> tuple[
        torch.Tensor, torch.Tensor, torch.Tensor]:
    """out[T,H], router_logits[T,E] (empty unless want_logits), aux[] for x[T,H]."""
    packed = _HANDLES[handle_id]
    h = packed.handle
    T, H = x.shape
    E = h.cfg.num_experts
    x = x.contiguous()
    out = torch.empty_like(x)
    aux = torch.empty((), dtype=torch.float32, device=x.device)
    logits = torch.empty((T, E) if want_logits else (0, E), dtype=torch.float32, device=x.device)
    ws = packed.workspace(T, x.device)
    stream = torch.cuda.current_stream(x.device).cuda_stream
    h.forward(x.data_ptr(), T, out.data_ptr(), logits.data_ptr() if want_logits else None,
              None, None, None, aux.data_ptr(), ws.data_ptr(), ws.numel(), stream)
    return out, logits, aux


def _moe_forward_residual(x: torch.Tensor, handle_id: int, want_logits: bool) -> tuple[
        torch.Tensor, torch.Tensor, torch.Tensor]:
    """x + MoE(LayerNorm(x)) [T,H], router_logits[T,E] (empty unless want_logits), aux[]."""
    packed = _HANDLES[handle_id]
    h = packed.handle
    T, H = x.shape
    E = h.cfg.num_experts
    x = x.contiguous()
    out = torch.empty_like(x)
    aux = torch.empty((), dtype=torch.float32, device=x.device)
    logits = torch.empty((T, E) if want_logits else (0, E), dtype=torch.float32, device=x.device)
    ws = packed.workspace(T, x.device)
    stream = torch.cuda.current_stream(x.device).cuda_stream
    h.forward_residual(x.data_ptr(), T, out.data_ptr(), logits.data_ptr() if want_logits else None,
                       None, None, None, aux.data_ptr(), ws.data_ptr(), ws.numel(), stream)
    return out, logits, aux


# The bodies above are registered as custom ops (for torch.compile, export and the other
# tracers); an eager call on a plain tensor runs the body directly, skipping the
# dispatcher's overhead (about 15 us a call, a tenth of a decode-sized forward).
moe_forward_op = torch.library.custom_op("vesper_moe::forward", mutates_args=(),
                                         device_types="cuda")(_moe_forward)
moe_forward_residual_op = torch.library.custom_op(
    "vesper_moe::forward_residual", mutates_args=(), device_types="cuda")(_moe_forward_residual)


def _eager(x: torch.Tensor) -> bool:
    """Whether a call with input x may skip the registered op: a plain tensor, no tracer."""
    return type(x) is torch.Tensor and not torch.compiler.is_compiling()


@moe_forward_residual_op.register_fake
def _(x, handle_id, want_logits):
    T, _ = x.shape
    E = _HANDLES[handle_id].handle.cfg.num_experts if handle_id in _HANDLES else 1
    return (torch.empty_like(x), x.new_empty((T, E) if want_logits else (0, E), dtype=torch.float32),
            x.new_empty((), dtype=torch.float32))


@moe_forward_op.register_fake
def _(x, handle_id, want_logits):
    T, _ = x.shape
    E = _HANDLES[handle_id].handle.cfg.num_experts if handle_id in _HANDLES else 1
    return (torch.empty_like(x), x.new_empty((T, E) if want_logits else (0, E), dtype=torch.float32),
            x.new_empty((), dtype=torch.float32))


def _ffn(x: torch.Tensor, handle_id: int) -> torch.Tensor:
    """Dense FeedForward out[T,H] for x[T,H] through vmoe_ffn_forward."""
    packed = _HANDLES[handle_id]
    h = packed.handle
    T, _ = x.shape
    x = x.contiguous()
    out = torch.empty_like(x)
    n = ctypes.c_size_t()
    _lib.check(h.lib.vmoe_ffn_workspace_size(h.ptr, T, ctypes.byref(n)), h.ptr)
    if packed.ws is None or packed.ws.numel() < n.value:
        packed.ws = torch.empty(max(n.value, 256), dtype=torch.uint8, device=x.device)
    stream = torch.cuda.current_stream(x.device).cuda_stream
    _lib.check(h.lib.vmoe_ffn_forward(h.ptr, ctypes.c_void_p(x.data_ptr()), T,
                                      ctypes.c_void_p(out.data_ptr()),
                                      ctypes.c_void_p(packed.ws.data_ptr()), packed.ws.numel(),
                                      ctypes.c_void_p(stream)), h.ptr, "vmoe_ffn_forward")
    return out


ffn_op = torch.library.custom_op("vesper_moe::ffn", mutates_args=(), device_types="cuda")(_ffn)


@ffn_op.register_fake
def _(x, handle_id):
    return torch.empty_like(x)


def _param_grad(g: torch.Tensor, p: torch.Tensor) -> torch.Tensor:
    return g.to(p.dtype) if g.dtype != p.dtype else g


class _MoETrainFn(torch.autograd.Function):
    """Autograd of the MoE layer through vmoe_forward_train / vmoe_backward (bf16)."""

    @staticmethod
    def forward(ctx, x2d, handle_id, layer, want_logits, *params):
        packed = _HANDLES[handle_id]
        h = packed.handle
        T, _ = x2d.shape
        dev = x2d.device
        saved_b, scratch_b = h.train_workspace_size(T)
        saved = torch.empty(max(saved_b, 256), dtype=torch.uint8, device=dev)
        out = torch.empty_like(x2d)
        aux = torch.empty((), dtype=torch.float32, device=dev)
        E = layer.config.moe_num_experts
        logits = torch.empty((T, E) if want_logits else (0, E), dtype=torch.float32, device=dev)
        stream = torch.cuda.current_stream(dev).cuda_stream
        h.forward_train(x2d.data_ptr(), T, out.data_ptr(), logits.data_ptr() if want_logits else None,
                        aux.data_ptr(), saved.data_ptr(), saved.numel(), stream)
        ctx.save_for_backward(x2d, saved)
        ctx.handle_id, ctx.layer, ctx.scratch_b = handle_id, layer, scratch_b
        ctx.mark_non_differentiable(logits)
        return out, aux, logits

    @staticmethod
    def backward(ctx, dout, daux, dlogits):
        x2d, saved = ctx.saved_tensors
        layer = ctx.layer
        h = _HANDLES[ctx.handle_id].handle
        dev = x2d.device
        T, H = x2d.shape
        c = layer.config
        E, I = c.moe_num_experts, c.intermediate_size
        if dout is None:
            dout = torch.zeros_like(x2d)
        dout = dout.to(x2d.dtype).contiguous()
        daux_t = (daux if daux is not None else torch.zeros((), device=dev)).float().reshape(1).contiguous()
        f = dict(device=dev, dtype=torch.float32)
        g = {"router_w": torch.empty(E, H, **f), "router_b": torch.empty(E, **f),
             "gate_w": torch.empty(E, I, H, **f), "gate_b": torch.empty(E, I, **f),
             "up_w": torch.empty(E, I, H, **f), "up_b": torch.empty(E, I, **f),
             "down_w": torch.empty(E, H, I, **f), "down_b": torch.empty(E, H, **f)}
        dx = torch.empty_like(x2d)
        scratch = torch.empty(max(ctx.scratch_b, 256), dtype=torch.uint8, device=dev)
        vg = _lib.VmoeGrads(**{k: ctypes.c_void_p(v.data_ptr()) for k, v in g.items()})
        stream = torch.cuda.current_stream(dev).cuda_stream
        h.backward(x2d.data_ptr(), dout.data_ptr(), T, daux_t.data_ptr(), dx.data_ptr(), vg,
                   saved.data_ptr(), saved.numel(), scratch.data_ptr(), scratch.numel(), stream)
        # FlyLoRA factors from the effective-weight gradients (W_eff = W + s U D,
        # b_eff = b + s (U b_D + b_U)): dU = s (dW D^T + db b_D^T), db_U = s db,
        # dD = s U^T dW, db_D = s U^T db
        s = c.lora_scaling
        lora = {}
        for name, attr in (("gate", "gate_proj"), ("up", "up_proj")):
            dW, db = g[f"{name}_w"], g[f"{name}_b"]
            U = torch.stack([getattr(e, attr).lora_up.weight.detach() for e in layer.experts]).float()
            D = torch.stack([getattr(e, attr).lora_down.weight.detach() for e in layer.experts]).float()
            bD = torch.stack([getattr(e, attr).lora_down.bias.detach() for e in layer.experts]).float()
            lora[name] = {
                "up_w": s * (torch.bmm(dW, D.transpose(1, 2)) + db[:, :, None] * bD[:, None, :]),
                "up_b": s * db,
                "down_w": s * torch.bmm(U.transpose(1, 2), dW),
                "down_b": s * torch.bmm(U.transpose(1, 2), db[:, :, None])[..., 0],
            }
        grads = [g["router_w"], g["router_b"]]
        for e in range(E):
            for name in ("gate", "up"):
                grads += [g[f"{name}_w"][e], g[f"{name}_b"][e], lora[name]["down_w"][e],
                          lora[name]["down_b"][e], lora[name]["up_w"][e], lora[name]["up_b"][e]]
            grads += [g["down_w"][e], g["down_b"][e]]
        params = layer._train_params()
        return (dx, None, None, None, *[_param_grad(gr, p) for gr, p in zip(grads, params)])


class _PackedHandleMixin:
    """Repack-on-change handle management shared by the MoE and dense layers."""

    def _param_list(self) -> list:
        """self.parameters() as a list, rebuilt only after a structural change."""
        cache = self.__dict__.get("_plist_cache")
        if cache is None or cache[0] != _STRUCTURE_GEN[0]:
            for m in self.modules():  # reassignments on these now invalidate the list
                _OWNED.add(m)
            cache = (_STRUCTURE_GEN[0], list(self.parameters()))
            self.__dict__["_plist_cache"] = cache
        return cache[1]

    def _weight_key(self):
        plist = self._param_list()
        pairs = (_native_pairs(plist) if _native_pairs is not None
                 else tuple((p.data_ptr(), p._version) for p in plist))
        return (_WRITE_GEN[0], self.__dict__.get("_dirty", 0), pairs)

    def mark_weights_dirty(self) -> None:
        """Repack the weights before the next forward.

        Needed only after writing parameters in a way the layer cannot see: through
        ``p.data`` (or a raw device pointer) outside a torch optimizer's ``step``.  Writes
        through the parameter itself (``with torch.no_grad(): p.copy_(...)``,
        ``load_state_dict``) and every ``torch.optim.Optimizer.step`` are detected.
        """
        self.__dict__["_dirty"] = self.__dict__.get("_dirty", 0) + 1

    def _abi_config(self, dtype: torch.dtype) -> _lib.VmoeConfig:
        c = self.config
        return _lib.VmoeConfig(hidden=c.hidden_size, inter=c.intermediate_size,
                               num_experts=c.moe_num_experts, top_k=c.moe_top_k,
                               lora_rank=c.flylora_rank, lora_scaling=c.lora_scaling,
                               era_gamma=c.era_gamma, dtype=_DTYPES[dtype],
                               capacity=c.moe_capacity)

    def packed_for(self, device: torch.device, dtype: torch.dtype) -> _Packed:
        """The handle for (device, dtype), repacking if any parameter changed."""
        if dtype not in _DTYPES:
            raise TypeError(f"vesper_moe supports float32 and bfloat16 inputs, not {dtype}")
        if device.type != "cuda":
            raise RuntimeError(f"velvetoptimizer_b200.{type(self).__name__} runs on CUDA tensors "
                               "only (there is no CPU path)")
        dev = device.index if device.index is not None else torch.cuda.current_device()
        slot = (dev, dtype)
        key = self._weight_key()
        packed = self._packed.get(slot)
        if packed is not None and packed.key == key:
            return packed
        if packed is None:
            packed = _Packed(self._new_handle(self._abi_config(dtype), dev), key)
            self._packed[slot] = packed
        with torch.cuda.device(dev):
            w = {k: v.to(device) for k, v in self.stacked_weights(dtype).items()}
            vw = _lib.VmoeWeights(**{k: ctypes.c_void_p(v.data_ptr()) for k, v in w.items()})
            stream = torch.cuda.current_stream(dev)
            packed.handle.set_weights(vw, stream.cuda_stream)
            # the stacked temporaries must outlive the enqueued copies
            stream.synchronize()
        packed.key = key
        return packed

    def close(self) -> None:
        for p in self._packed.values():
            p.release()
        self._packed.clear()


class FeedForward(_PackedHandleMixin, nn.Module):
    """Drop-in for the reference dense FeedForward (python/vesper/model.py:249-270).

    Same submodule names (``gate_proj``/``up_proj`` FlyLoRA linears, ``down_proj``), so the
    reference's state_dict loads unchanged; ``forward(x[..., H]) -> out[..., H]``.  It runs
    on the same grouped tensor-core GEMMs as the MoE experts (one expert, no router).
    """

    def __init__(self, config):
        _install_hooks()
        super().__init__()
        cfg = MoEConfig.from_any(config)
        self.config = cfg
        args = (cfg.hidden_size, cfg.intermediate_size, cfg.flylora_rank, cfg.flylora_alpha,
                cfg.flylora_sparsity)
        self.gate_proj = FlyLoRALinear(*args)
        self.up_proj = FlyLoRALinear(*args)
        self.down_proj = nn.Linear(cfg.intermediate_size, cfg.hidden_size)
        self._packed: dict[tuple, _Packed] = {}

    def _new_handle(self, abi, dev):
        return _lib.Handle(abi, dev, dense=True)

    def stacked_weights(self, dtype: torch.dtype) -> dict[str, torch.Tensor]:
        def one(t):
            return t.detach().to(dtype).unsqueeze(0).contiguous()

        w = {}
        for name, mod in (("gate", self.gate_proj), ("up", self.up_proj)):
            w[f"{name}_w"], w[f"{name}_b"] = one(mod.base.weight), one(mod.base.bias)
            w[f"{name}_lora_down_w"] = one(mod.lora_down.weight)
            w[f"{name}_lora_down_b"] = one(mod.lora_down.bias)
            w[f"{name}_lora_up_w"] = one(mod.lora_up.weight)
            w[f"{name}_lora_up_b"] = one(mod.lora_up.bias)
        w["down_w"], w["down_b"] = one(self.down_proj.weight), one(self.down_proj.bias)
        return w

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        shape = x.shape
        packed = self.packed_for(x.device, x.dtype)
        x2d = x.reshape(-1, shape[-1])
        out = _ffn(x2d, packed.id) if _eager(x2d) else torch.ops.vesper_moe.ffn(x2d, packed.id)
        return out.reshape(shape)


# ---------------------------------------------------------------------------------------
# the layer
# ---------------------------------------------------------------------------------------
class MoELayer(_PackedHandleMixin, nn.Module):
    """Mixture of Experts with top-K routing and the Switch load-balancing loss.

    Same constructor argument (a VesperConfig-like object), parameters, state_dict keys
    and ``forward`` contract as the reference ``MoELayer``.
    """

    def __init__(self, config):
        _install_hooks()
        super().__init__()
        cfg = MoEConfig.from_any(config)
        cfg.validate()
        self.config = cfg
        self.num_experts = cfg.moe_num_experts
        self.top_k = cfg.moe_top_k
        self.aux_loss_weight = cfg.moe_aux_loss_weight
        self.router = nn.Linear(cfg.hidden_size, cfg.moe_num_experts)
        self.experts = nn.ModuleList([ExpertFFN(cfg) for _ in range(cfg.moe_num_experts)])
        self._packed: dict[tuple, _Packed] = {}

    # -- weights ---------------------------------------------------------------------
    def _new_handle(self, abi, dev):
        return _lib.Handle(abi, dev)

    def stacked_weights(self, dtype: torch.dtype) -> dict[str, torch.Tensor]:
        """The per-expert parameters stacked on a leading expert axis, in ``dtype``."""
        ex = self.experts

        def st(get):
            return torch.stack([get(e).detach() for e in ex]).to(dtype).contiguous()

        w = {"router_w": self.router.weight.detach().to(dtype).contiguous(),
             "router_b": self.router.bias.detach().to(dtype).contiguous()}
        for name, attr in (("gate", "gate_proj"), ("up", "up_proj")):
            w[f"{name}_w"] = st(lambda e: getattr(e, attr).base.weight)
            w[f"{name}_b"] = st(lambda e: getattr(e, attr).base.bias)
            w[f"{name}_lora_down_w"] = st(lambda e: getattr(e, attr).lora_down.weight)
            w[f"{name}_lora_down_b"] = st(lambda e: getattr(e, attr).lora_down.bias)
            w[f"{name}_lora_up_w"] = st(lambda e: getattr(e, attr).lora_up.weight)
            w[f"{name}_lora_up_b"] = st(lambda e: getattr(e, attr).lora_up.bias)
        w["down_w"] = st(lambda e: e.down_proj.weight)
        w["down_b"] = st(lambda e: e.down_proj.bias)
        return w

    def _train_params(self) -> list:
        """The parameters in the order the training autograd Function takes them."""
        ps = [self.router.weight, self.router.bias]
        for e in self.experts:
            for proj in (e.gate_proj, e.up_proj):
                ps += [proj.base.weight, proj.base.bias, proj.lora_down.weight,
                       proj.lora_down.bias, proj.lora_up.weight, proj.lora_up.bias]
            ps += [e.down_proj.weight, e.down_proj.bias]
        return ps

    def _wants_grad(self, x: torch.Tensor) -> bool:
        return torch.is_grad_enabled() and (
            x.requires_grad or any(p.requires_grad for p in self._param_list()))

    # -- forward ---------------------------------------------------------------------
    def forward(self, x: torch.Tensor, return_router_logits: bool = False):
        """(out[B,S,H], aux_loss[]) — or (out, aux_loss, router_logits[B,S,E])."""
        B, S, H = x.shape
        packed = self.packed_for(x.device, x.dtype)
        if self._wants_grad(x):
            if x.dtype == torch.bfloat16:
                if not getattr(packed, "training", False):
                    packed.handle.set_training(True, torch.cuda.current_stream(x.device).cuda_stream)
                    packed.training = True
                out, aux, logits = _MoETrainFn.apply(
                    x.reshape(B * S, H).contiguous(), packed.id, self, bool(return_router_logits),
                    *self._train_params())
                out = out.reshape(B, S, H)
                if return_router_logits:
                    return out, aux, logits.reshape(B, S, self.num_experts)
                return out, aux
            if not getattr(self, "_warned_fp32_grad", False):
                warnings.warn("velvetoptimizer_b200.MoELayer: the backward runs on bfloat16 "
                              "inputs; this float32 forward carries no gradient")
                self._warned_fp32_grad = True
        x2d = x.reshape(B * S, H)
        op = _moe_forward if _eager(x2d) else torch.ops.vesper_moe.forward
        out, logits, aux = op(x2d, packed.id, bool(return_router_logits))
        out = out.reshape(B, S, H)
        if return_router_logits:
            return out, aux, logits.reshape(B, S, self.num_experts)
        return out, aux

    def forward_residual(self, hidden_states: torch.Tensor, norm: nn.LayerNorm,
                         return_router_logits: bool = False):
        """The FFN half of the reference's pre-norm TransformerLayer.forward in one call:
        ``(hidden_states + self(norm(hidden_states))[0], aux_loss)`` (python/vesper/model.py
        :418-425), with the LayerNorm folded into the router's and the dispatch's reads and
        the residual add into the combine (``vmoe_forward_residual``).  ``norm`` is the
        layer's ``ffn_norm`` (an ``nn.LayerNorm`` over hidden_size)."""
        B, S, H = hidden_states.shape
        if not isinstance(norm, nn.LayerNorm) or tuple(norm.normalized_shape) != (H,):
            raise ValueError("norm must be an nn.LayerNorm over the hidden size")
        x = hidden_states
        packed = self.packed_for(x.device, x.dtype)
        key = (tuple((p.data_ptr(), p._version) for p in norm.parameters()), float(norm.eps),
               packed.key)
        if getattr(packed, "norm_key", None) != key:
            dev = x.device
            with torch.cuda.device(dev):
                w = norm.weight.detach().to(dev, x.dtype).contiguous() if norm.weight is not None else None
                b = norm.bias.detach().to(dev, x.dtype).contiguous() if norm.bias is not None else None
                stream = torch.cuda.current_stream(dev)
                packed.handle.set_norm(_ptr(w), _ptr(b), norm.eps, stream.cuda_stream)
                stream.synchronize()  # the converted parameters must outlive the enqueued copy
            packed.norm_key = key
        x2d = x.reshape(B * S, H)
        op = _moe_forward_residual if _eager(x2d) else torch.ops.vesper_moe.forward_residual
        out, logits, aux = op(x2d, packed.id, bool(return_router_logits))
        out = out.reshape(B, S, H)
        if return_router_logits:
            return out, aux, logits.reshape(B, S, self.num_experts)
        return out, aux

    def forward_host(self, x: torch.Tensor, device=None, chunks: int = 0,
                     out: torch.Tensor | None = None):
        """``forward`` for x[B,S,H] in host memory, computed on a CUDA device.

        The reference runs a CPU tensor through the layer on the CPU; here the batch goes
        to ``device`` (default: the current CUDA device) in token chunks whose host->device
        copy, layer forward and device->host copy overlap (``vmoe_forward_host``).  x and
        ``out`` should be pinned (``pin_memory()``) for the copies to overlap.  Returns
        (out[B,S,H], aux_loss[]) as host tensors, ready on return; out is bit-identical to
        ``forward`` of the same tokens.
        """
        if x.device.type != "cpu":
            raise ValueError("forward_host takes a host tensor; use forward for CUDA tensors")
        B, S, H = x.shape
        if device is None:
            device = torch.device("cuda", torch.cuda.current_device())
        device = torch.device(device)
        packed = self.packed_for(device, x.dtype)
        x = x.contiguous()
        if out is None:
            out = torch.empty(x.shape, dtype=x.dtype, pin_memory=x.is_pinned())
        elif out.shape != x.shape or out.dtype != x.dtype or out.device.type != "cpu" \
                or not out.is_contiguous():
            raise ValueError("out must be a contiguous host tensor shaped and typed like x")
        aux = torch.empty((), dtype=torch.float32, pin_memory=True)
        T = B * S
        h = packed.handle
        with torch.cuda.device(device):
            ws = packed.scratch(h.host_workspace_size(T, chunks), device)
            stream = torch.cuda.current_stream(device)
            h.forward_host(x.data_ptr(), T, out.data_ptr(), aux.data_ptr(), int(chunks),
                           ws.data_ptr(), ws.numel(), stream.cuda_stream)
            stream.synchronize()
        return out, aux
