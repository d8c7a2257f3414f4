"""Expert-parallel MoE layer: experts sharded over the ranks of a process group.

The reference has no distributed code; the path's specification partitions the MoE layer
expert-parallel over one 8-GPU NVLink box with NCCL all-to-all dispatch and combine.  With
G ranks, rank r holds experts [r*E/G, (r+1)*E/G) and routes its own tokens.  One forward:

1. ``vmoe_ep_route`` (CUDA): router over all E experts, each routed (token, k) row written
   to ``send_rows`` expert-major (hence destination-rank-major), and the per-expert counts;
2. counts all-to-all (NCCL), one device->host read of the counts;
3. rows all-to-all-v (NCCL point-to-point, one message per (peer, expert) chunk) into
   ``recv_rows``, whose per-local-expert segments are padded to 128-row GEMM tiles;
4. ``vmoe_ep_experts`` (CUDA): the local grouped gate|up (+ERA*up) and down GEMMs;
5. the reverse all-to-all-v of the expert outputs into ``back_rows``;
6. ``vmoe_ep_combine`` (CUDA): the deterministic fp32 combine.

A token's output is bit-identical to the single-GPU forward (same kernels per row, same
combine order).  The aux loss is that of this rank's tokens (``E * sum f_e P_e`` over them),
which is what the reference computes for the same batch.

``plan_exchange`` and ``exchange_rows`` are plain torch/numpy and backend-agnostic, so the
exchange logic is tested with gloo ranks on CPU.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np
import torch
import torch.distributed as dist

from . import _lib
from .config import MoEConfig

TILE_ROWS = 128


@dataclass
class ExchangePlan:
    send_offsets: np.ndarray   # [E+1] first send row of each global expert (unpadded)
    recv_counts: np.ndarray    # [G, El] rows rank s sends for each local expert
    recv_offsets: np.ndarray   # [G, El] first recv row of chunk (s, e)
    seg_offsets: np.ndarray    # [El+1] padded segment of each local expert in recv_rows
    recv_rows: int             # padded total, a multiple of 128
    tile_expert: np.ndarray    # [recv_rows / 128] local expert of each 128-row tile


def plan_exchange(send_counts, recv_counts, align: int = TILE_ROWS) -> ExchangePlan:
    """Row layout of both exchanges from this rank's counts.

    ``send_counts[E]``: rows this rank routes to each global expert.
    ``recv_counts[G, El]``: rows each source rank routes to each of this rank's experts.
    """
    send_counts = np.asarray(send_counts, dtype=np.int64)
    recv_counts = np.asarray(recv_counts, dtype=np.int64)
    G, El = recv_counts.shape
    send_offsets = np.zeros(len(send_counts) + 1, dtype=np.int64)
    np.cumsum(send_counts, out=send_offsets[1:])
    per_expert = recv_counts.sum(axis=0)
    padded = (per_expert + align - 1) // align * align
    seg_offsets = np.zeros(El + 1, dtype=np.int64)
    np.cumsum(padded, out=seg_offsets[1:])
    recv_offsets = np.zeros((G, El), dtype=np.int64)
    for e in range(El):
        recv_offsets[:, e] = seg_offsets[e] + np.concatenate(([0], np.cumsum(recv_counts[:-1, e])))
    total = int(seg_offsets[-1])
    tile_expert = np.repeat(np.arange(El, dtype=np.int32), padded // align)
    return ExchangePlan(send_offsets, recv_counts, recv_offsets, seg_offsets, total, tile_expert)


def exchange_rows(src: torch.Tensor, dst: torch.Tensor, plan: ExchangePlan, rank: int,
                  world: int, reverse: bool = False, group=None) -> None:
    """All-to-all-v of rows between the send layout and the recv layout of ``plan``.

    Chunk (peer, e) pairs this rank's rows for global expert ``peer*El + e`` (send layout,
    ``send_offsets``) with ``peer``'s rows for this rank's local expert ``e`` (recv layout,
    ``recv_offsets``).  Forward: send-layout ``src`` -> recv-layout ``dst``; reverse: the
    opposite.  Between one pair of ranks the messages go in ascending local-expert order on
    both sides, so point-to-point matching pairs them; empty chunks are skipped on both
    sides (both know the count); this rank's own chunks are device-local copies.
    """
    El = plan.recv_counts.shape[1]
    send_cnt = np.diff(plan.send_offsets)
    ops = []
    for peer in range(world):
        gpeer = peer if group is None else dist.get_global_rank(group, peer)
        for e in range(El):
            g = peer * El + e
            mine = (int(plan.send_offsets[g]), int(send_cnt[g]))                  # send layout
            theirs = (int(plan.recv_offsets[peer, e]), int(plan.recv_counts[peer, e]))  # recv layout
            out_chunk, in_chunk = (mine, theirs) if not reverse else (theirs, mine)
            if peer == rank:  # this rank's own rows: a device-local copy
                (so, n), (do, _) = out_chunk, in_chunk
                if n:
                    dst[do:do + n].copy_(src[so:so + n])
                continue
            if out_chunk[1]:
                ops.append(dist.P2POp(dist.isend, src[out_chunk[0]:out_chunk[0] + out_chunk[1]],
                                      gpeer, group))
            if in_chunk[1]:
                ops.append(dist.P2POp(dist.irecv, dst[in_chunk[0]:in_chunk[0] + in_chunk[1]],
                                      gpeer, group))
    if ops:
        for req in dist.batch_isend_irecv(ops):
            req.wait()


class ExpertParallelMoE:
    """The MoE layer with its experts sharded over ``group`` (default: the world group).

    ``weights`` holds the GLOBAL stacked tensors of ``MoELayer.stacked_weights`` (router
    ``[E, H]``, experts ``[E, ...]``); each rank keeps the router and its own slice.

    ``transport``:
      * ``"p2p"`` (default) -- the exchange runs inside the kernels over NVLink peer memory
        (``vmoe_ep_p2p_forward``): one call per forward, no host synchronisation; every rank
        must call ``forward`` the same number of times with at most ``max_tokens`` tokens;
        ``chunks`` token chunks run on internal streams so that the NVLink traffic of one
        overlaps the GEMMs of another;
      * ``"nccl"`` -- the staged path: route, NCCL all-to-all-v, experts, all-to-all-v back,
        combine.
    """

    def __init__(self, config, weights: dict[str, torch.Tensor], device: torch.device,
                 dtype: torch.dtype = torch.bfloat16, group=None, transport: str = "p2p",
                 max_tokens: int | None = None, chunks: int = 2):
        cfg = MoEConfig.from_any(config)
        cfg.validate()
        self.cfg, self.group, self.device, self.dtype = cfg, group, device, dtype
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        E = cfg.moe_num_experts
        if E % self.world:
            raise ValueError(f"{E} experts do not shard over {self.world} ranks")
        self.E, self.El, self.K, self.H = E, E // self.world, cfg.moe_top_k, cfg.hidden_size
        abi = _lib.VmoeConfig(hidden=cfg.hidden_size, inter=cfg.intermediate_size,
                              num_experts=E, top_k=cfg.moe_top_k, lora_rank=cfg.flylora_rank,
                              lora_scaling=cfg.lora_scaling, era_gamma=cfg.era_gamma,
                              dtype=_lib.VMOE_F32 if dtype == torch.float32 else _lib.VMOE_BF16,
                              capacity=0)
        self.lib = _lib.load()
        self.h = ctypes.c_void_p()
        dev = device.index if device.index is not None else torch.cuda.current_device()
        _lib.check(self.lib.vmoe_create_ep(ctypes.byref(abi), dev, self.world, self.rank,
                                           ctypes.byref(self.h)), None, "vmoe_create_ep")
        lo, hi = self.rank * self.El, (self.rank + 1) * self.El
        local = {}
        for k, v in weights.items():
            v = v.to(device=device, dtype=dtype)
            local[k] = (v if k.startswith("router") else v[lo:hi]).contiguous()
        vw = _lib.VmoeWeights(**{k: ctypes.c_void_p(t.data_ptr()) for k, t in local.items()})
        stream = torch.cuda.current_stream(device)
        _lib.check(self.lib.vmoe_set_weights(self.h, ctypes.byref(vw), ctypes.c_void_p(stream.cuda_stream)),
                   self.h, "vmoe_set_weights")
        stream.synchronize()
        self.last_plan: ExchangePlan | None = None
        self.launches = 0
        if transport not in ("p2p", "nccl"):
            raise ValueError(f"transport must be 'p2p' or 'nccl', not {transport!r}")
        self.transport = transport
        self.max_tokens = max_tokens
        self._p2p_ws = None
        self._host_ws = None
        if transport == "p2p":
            if max_tokens is None:
                raise ValueError("transport='p2p' needs max_tokens (tokens per rank per forward)")
            caps = [None] * self.world
            dist.all_gather_object(caps, int(max_tokens), group=group)
            if len(set(caps)) != 1:  # the symmetric regions must have one layout
                raise ValueError(f"max_tokens differs across ranks: {caps}")
            self.chunks = int(chunks)
            handle = ctypes.create_string_buffer(64 * self.chunks)
            _lib.check(self.lib.vmoe_ep_p2p_setup(self.h, int(max_tokens), self.chunks, handle),
                       self.h, "vmoe_ep_p2p_setup")
            handles = [None] * self.world
            dist.all_gather_object(handles, handle.raw, group=group)
            blob = ctypes.create_string_buffer(b"".join(handles), 64 * self.chunks * self.world)
            _lib.check(self.lib.vmoe_ep_p2p_connect(self.h, blob), self.h, "vmoe_ep_p2p_connect")
            dist.barrier(group=group)
        # set to a list to record (stage -> (start, end) CUDA events) for every forward
        self.stage_events: list[dict] | None = None

    def _ws(self, tokens: int, rows: int) -> torch.Tensor:
        n = ctypes.c_size_t()
        _lib.check(self.lib.vmoe_ep_workspace_size(self.h, tokens, rows, ctypes.byref(n)), self.h)
        return torch.empty(max(n.value, 256), dtype=torch.uint8, device=self.device)

    def _mark(self, rec: dict | None, name: str):
        if rec is not None:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record(torch.cuda.current_stream(self.device))
            rec.setdefault("_order", []).append((name, ev))

    def forward(self, x: torch.Tensor):
        """x [T, H] on this rank -> (out [T, H], aux_loss of this rank's tokens)."""
        if self.transport == "p2p":
            return self._forward_p2p(x)
        return self._forward_nccl(x)

    def _forward_p2p(self, x: torch.Tensor):
        lib, h, dev = self.lib, self.h, self.device
        T, H = x.shape
        x = x.contiguous()
        n = ctypes.c_size_t()
        _lib.check(lib.vmoe_ep_p2p_workspace_size(h, T, ctypes.byref(n)), h)
        if self._p2p_ws is None or self._p2p_ws.numel() < n.value:
            self._p2p_ws = torch.empty(max(n.value, 256), dtype=torch.uint8, device=dev)
        out = torch.empty_like(x)
        aux = torch.empty((), dtype=torch.float32, device=dev)
        stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
        _lib.check(lib.vmoe_ep_p2p_forward(h, ctypes.c_void_p(x.data_ptr()), T,
                                           ctypes.c_void_p(out.data_ptr()), None,
                                           ctypes.c_void_p(aux.data_ptr()),
                                           ctypes.c_void_p(self._p2p_ws.data_ptr()),
                                           self._p2p_ws.numel(), stream), h, "vmoe_ep_p2p_forward")
        self.launches = lib.vmoe_last_launch_count(h)
        return out, aux

    def forward_host(self, x: torch.Tensor, out: torch.Tensor | None = None):
        """``forward`` for x [T, H] in host memory (fused NVLink transport): each token
        chunk's rows are copied to this rank's GPU, run and copied back with the copies
        overlapping the other chunks (``vmoe_ep_p2p_forward_host``).  x and ``out`` should
        be pinned.  Returns (out [T, H], aux_loss) as host tensors, ready on return; out is
        bit-identical to ``forward`` of the same tokens."""
        if self.transport != "p2p":
            raise ValueError("forward_host runs on the fused NVLink transport ('p2p')")
        if x.device.type != "cpu":
            raise ValueError("forward_host takes a host tensor; use forward for CUDA tensors")
        lib, h, dev = self.lib, self.h, self.device
        T, H = x.shape
        x = x.contiguous()
        if out is None:
            out = torch.empty(x.shape, dtype=x.dtype, pin_memory=x.is_pinned())
        elif out.shape != x.shape or out.dtype != x.dtype or out.device.type != "cpu" \
                or not out.is_contiguous():
            raise ValueError("out must be a contiguous host tensor shaped and typed like x")
        n = ctypes.c_size_t()
        _lib.check(lib.vmoe_ep_p2p_host_workspace_size(h, ctypes.byref(n)), h)
        if self._host_ws is None or self._host_ws.numel() < n.value:
            self._host_ws = torch.empty(max(n.value, 256), dtype=torch.uint8, device=dev)
        aux = torch.empty((), dtype=torch.float32, pin_memory=True)
        stream = torch.cuda.current_stream(dev)
        _lib.check(lib.vmoe_ep_p2p_forward_host(h, ctypes.c_void_p(x.data_ptr()), T,
                                                ctypes.c_void_p(out.data_ptr()),
                                                ctypes.c_void_p(aux.data_ptr()),
                                                ctypes.c_void_p(self._host_ws.data_ptr()),
                                                self._host_ws.numel(),
                                                ctypes.c_void_p(stream.cuda_stream)),
                   h, "vmoe_ep_p2p_forward_host")
        self.launches = lib.vmoe_last_launch_count(h)
        stream.synchronize()
        return out, aux

    def set_profiling(self, forwards: int) -> None:
        _lib.check(self.lib.vmoe_set_profiling(self.h, int(forwards)), self.h)

    def stage_times(self):
        buf = (ctypes.c_float * 16)()
        n, f = ctypes.c_int(), ctypes.c_int()
        _lib.check(self.lib.vmoe_stage_times(self.h, buf, 16, ctypes.byref(n), ctypes.byref(f)), self.h)
        return {self.lib.vmoe_stage_name(i).decode(): float(buf[i]) for i in range(n.value)}, f.value

    def device_status(self) -> int:
        """The device status word (0 = fine; timeouts and bad-index codes otherwise); clears it."""
        code = ctypes.c_int32()
        rc = self.lib.vmoe_device_status(self.h, ctypes.byref(code),
                                         ctypes.c_void_p(torch.cuda.current_stream(self.device).cuda_stream))
        if rc not in (_lib.VMOE_OK, _lib.VMOE_ERR_TIMEOUT, _lib.VMOE_ERR_DEVICE_STATUS):
            _lib.check(rc, self.h, "vmoe_device_status")
        return code.value

    def _forward_nccl(self, x: torch.Tensor):
        lib, h, dev = self.lib, self.h, self.device
        rec = {} if self.stage_events is not None else None
        self._mark(rec, "route")
        T, H = x.shape
        x = x.contiguous()
        stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
        send = torch.empty((T * self.K, H), dtype=self.dtype, device=dev)
        counts = torch.empty((self.E,), dtype=torch.int32, device=dev)
        aux = torch.empty((), dtype=torch.float32, device=dev)
        ws = self._ws(T, 0)
        _lib.check(lib.vmoe_ep_route(h, ctypes.c_void_p(x.data_ptr()), T,
                                     ctypes.c_void_p(send.data_ptr()),
                                     ctypes.c_void_p(counts.data_ptr()), None,
                                     ctypes.c_void_p(aux.data_ptr()),
                                     ctypes.c_void_p(ws.data_ptr()), ws.numel(), stream),
                   h, "vmoe_ep_route")
        launches = lib.vmoe_last_launch_count(h)
        self._mark(rec, "exchange_counts_rows")
        # counts: mine for every expert, and every rank's for my experts
        recv_counts = torch.empty((self.world * self.El,), dtype=torch.int32, device=dev)
        dist.all_to_all_single(recv_counts, counts, group=self.group)
        both = torch.cat([counts, recv_counts]).cpu().numpy().astype(np.int64)
        plan = plan_exchange(both[:self.E], both[self.E:].reshape(self.world, self.El),
                             align=int(lib.vmoe_gemm_tile_rows(h)))
        self.last_plan = plan
        rows = plan.recv_rows
        recv = torch.empty((rows, H), dtype=self.dtype, device=dev)
        exchange_rows(send, recv, plan, self.rank, self.world, group=self.group)
        y = torch.empty((rows, H), dtype=self.dtype, device=dev)
        self._mark(rec, "experts_gemm1_gemm2")
        if rows:
            tiles = torch.from_numpy(plan.tile_expert).to(dev, non_blocking=True)
            ntiles = torch.tensor([len(plan.tile_expert)], dtype=torch.int32).to(dev, non_blocking=True)
            ws2 = self._ws(0, rows)
            _lib.check(lib.vmoe_ep_experts(h, ctypes.c_void_p(recv.data_ptr()), rows,
                                           ctypes.c_void_p(tiles.data_ptr()),
                                           ctypes.c_void_p(ntiles.data_ptr()),
                                           ctypes.c_void_p(y.data_ptr()),
                                           ctypes.c_void_p(ws2.data_ptr()), ws2.numel(), stream),
                       h, "vmoe_ep_experts")
            launches += lib.vmoe_last_launch_count(h)
        back = torch.empty_like(send)
        self._mark(rec, "exchange_back")
        exchange_rows(y, back, plan, self.rank, self.world, reverse=True, group=self.group)
        out = torch.empty_like(x)
        self._mark(rec, "combine")
        _lib.check(lib.vmoe_ep_combine(h, ctypes.c_void_p(back.data_ptr()), T,
                                       ctypes.c_void_p(out.data_ptr()),
                                       ctypes.c_void_p(ws.data_ptr()), ws.numel(), stream),
                   h, "vmoe_ep_combine")
        self.launches = launches + lib.vmoe_last_launch_count(h)
        self._mark(rec, "end")
        if rec is not None:
            rec["recv_rows_real"] = int(plan.recv_counts.sum())
            self.stage_events.append(rec)
        return out, aux

    @staticmethod
    def stage_ms(records: list[dict]) -> dict[str, float]:
        """Average milliseconds per stage over recorded forwards (synchronises)."""
        acc: dict[str, float] = {}
        for rec in records:
            order = rec["_order"]
            order[-1][1].synchronize()
            for (name, a), (_, b) in zip(order[:-1], order[1:]):
                acc[name] = acc.get(name, 0.0) + a.elapsed_time(b)
        return {k: v / max(1, len(records)) for k, v in acc.items()}

    __call__ = forward

    def close(self):
        """Free this rank's handle.  Collective: peers may still be reading this rank's
        expert outputs (or writing its receive buffer) until every rank is done, so all
        ranks synchronise their devices and meet at a barrier before anything is freed."""
        if self.h:
            torch.cuda.synchronize(self.device)
            dist.barrier(group=self.group)
            self.lib.vmoe_destroy(self.h)
            self.h = ctypes.c_void_p()
