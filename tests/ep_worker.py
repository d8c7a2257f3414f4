"""Expert-parallel parity worker: run under torchrun, one rank per GPU.

    torchrun --nproc-per-node N --master-addr 127.0.0.1 --master-port P tests/ep_worker.py

Every rank builds the same global weights, routes its own tokens through the
expert-parallel layer (experts sharded over the ranks, NCCL exchange) and through the
single-GPU forward with all experts, and requires the outputs to be bit-identical (the same
kernels compute each row and the combine order is fixed); the fused transport's host-buffer
forward must reproduce its device forward bit for bit.  Exit code 0 on success.
"""
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from velvetoptimizer_b200 import MoEConfig, _lib  # noqa: E402
from velvetoptimizer_b200.ep import ExpertParallelMoE  # noqa: E402


def global_weights(cfg, device, dtype, seed=0):
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    E, H, I, r = cfg.moe_num_experts, cfg.hidden_size, cfg.intermediate_size, cfg.flylora_rank
    n = lambda *s: (torch.randn(*s, generator=g, device=device) * 0.02).to(dtype)  # noqa: E731
    b = lambda *s: (torch.randn(*s, generator=g, device=device) * 0.01).to(dtype)  # noqa: E731
    w = {"router_w": n(E, H), "router_b": b(E), "down_w": n(E, H, I), "down_b": b(E, H)}
    for p in ("gate", "up"):
        w[f"{p}_w"], w[f"{p}_b"] = n(E, I, H), b(E, I)
        w[f"{p}_lora_down_w"], w[f"{p}_lora_down_b"] = n(E, r, H), b(E, r)
        w[f"{p}_lora_up_w"], w[f"{p}_lora_up_b"] = n(E, I, r), b(E, I)
    return w


def single_gpu(cfg, w, x, dtype):
    abi = _lib.VmoeConfig(hidden=cfg.hidden_size, inter=cfg.intermediate_size,
                          num_experts=cfg.moe_num_experts, top_k=cfg.moe_top_k,
                          lora_rank=cfg.flylora_rank, lora_scaling=cfg.lora_scaling,
                          era_gamma=cfg.era_gamma,
                          dtype=_lib.VMOE_F32 if dtype == torch.float32 else _lib.VMOE_BF16,
                          capacity=0)
    h = _lib.Handle(abi, x.device.index)
    import ctypes
    h.set_weights(_lib.VmoeWeights(**{k: ctypes.c_void_p(v.data_ptr()) for k, v in w.items()}),
                  torch.cuda.current_stream().cuda_stream)
    T = x.shape[0]
    ws = torch.empty(h.workspace_size(T), dtype=torch.uint8, device=x.device)
    out = torch.empty_like(x)
    aux = torch.empty((), dtype=torch.float32, device=x.device)
    h.forward(x.data_ptr(), T, out.data_ptr(), None, None, None, None, aux.data_ptr(),
              ws.data_ptr(), ws.numel(), torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    h.close()
    return out, aux


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    from datetime import timedelta
    dist.init_process_group("nccl", timeout=timedelta(seconds=60), device_id=dev)
    failures = []
    try:
        cases = [
            (torch.bfloat16, MoEConfig(hidden_size=512, intermediate_size=384, moe_num_experts=8,
                                       moe_top_k=2), 1000),
            (torch.bfloat16, MoEConfig(hidden_size=256, intermediate_size=256,
                                       moe_num_experts=4 * world, moe_top_k=4), 777),
            (torch.float32, MoEConfig(hidden_size=128, intermediate_size=192, moe_num_experts=8,
                                      moe_top_k=3), 300),
        ]
        # p2p: the default exchange (bf16 outputs pushed by the down GEMM's epilogue up to 2
        # ranks, pulled by the combine beyond); "push" / "pull" force either (VMOE_EP_PUSH),
        # so both run at any rank count (fp32 always pulls)
        for transport, chunks in (("nccl", 1), ("p2p", 1), ("p2p", 2), ("p2p", 3), ("pull", 2),
                                  ("push", 2)):
            for dtype, cfg, T0 in cases:
                T = T0 - 37 * rank  # ranks route different token counts
                if chunks == 3 and rank == world - 1:
                    T = 5  # this rank's later chunks are empty but still take part
                w = global_weights(cfg, dev, dtype, seed=7)
                if transport in ("pull", "push"):
                    os.environ["VMOE_EP_PUSH"] = "0" if transport == "pull" else "1"
                layer = ExpertParallelMoE(cfg, w, dev, dtype,
                                          transport="nccl" if transport == "nccl" else "p2p",
                                          max_tokens=T0, chunks=chunks)
                os.environ.pop("VMOE_EP_PUSH", None)
                tag = (f"{transport}x{chunks} rank {rank} {dtype} E{cfg.moe_num_experts} "
                       f"K{cfg.moe_top_k}")
                for it in range(3):  # several forwards: epochs advance, buffers are reused
                    g = torch.Generator(device=dev)
                    g.manual_seed(1000 + 10 * rank + it)
                    x = torch.randn(T, cfg.hidden_size, generator=g, device=dev).to(dtype)
                    out, aux = layer(x)
                    out2, aux2 = layer(x)
                    if transport != "nccl":  # the host-buffer forward (every rank calls it)
                        out_h, aux_h = layer.forward_host(x.cpu().pin_memory())
                    torch.cuda.synchronize()
                    status = layer.device_status()
                    if status:
                        failures.append(f"{tag}: device status 0x{status:x}")
                    ref, ref_aux = single_gpu(cfg, w, x, dtype)
                    if not torch.equal(out, ref):
                        d = (out.float() - ref.float()).abs().max().item()
                        failures.append(f"{tag} it{it}: EP output differs from single GPU (max abs {d:.3e})")
                    if not torch.equal(out, out2):
                        failures.append(f"{tag} it{it}: EP output not deterministic")
                    if transport != "nccl":
                        if not torch.equal(out_h, out.cpu()):
                            failures.append(f"{tag} it{it}: host-buffer EP output differs")
                        if abs(aux_h.item() - aux.item()) > 1e-6 * abs(aux.item()):
                            failures.append(f"{tag} it{it}: host-buffer aux {aux_h.item()} vs "
                                            f"{aux.item()}")
                    if (abs(aux.item() - ref_aux.item()) > 1e-6 * abs(ref_aux.item())
                            or aux.item() != aux2.item()):
                        failures.append(f"{tag} it{it}: aux {aux.item()} vs {ref_aux.item()}")
                if transport == "nccl":
                    rows = int(layer.last_plan.recv_counts.sum())
                    tot = torch.tensor([rows], device=dev)
                    dist.all_reduce(tot)
                    want = sum(T0 - 37 * r for r in range(world)) * cfg.moe_top_k
                    if int(tot.item()) != want:
                        failures.append(f"{tag}: {int(tot.item())} rows exchanged, want {want}")
                layer.close()
                dist.barrier()
    finally:
        dist.destroy_process_group()
    if failures:
        print("\n".join(failures), flush=True)
        return 1
    print(f"EP_OK rank {rank} of {world}", flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
