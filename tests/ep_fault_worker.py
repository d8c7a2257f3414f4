"""Failure detection of the fused expert-parallel forward, without any GPU fault.

Run under torchrun with 2 ranks (one GPU each).  Both ranks run one forward.  Then rank 1
stops launching work -- it stays alive on the host and launches nothing, like a rank that
stalls between steps -- while rank 0 runs a second forward.  Every spin in rank 0's kernels
is bounded, so that forward ends on its own; vmoe_device_status must report the peer-wait
timeout, and rank 0's CUDA context must still work: a single-GPU forward afterwards must
reproduce the first, healthy, expert-parallel output bit for bit.  Exit code 0 on success.
"""
import os
import sys
import time

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))

from ep_worker import global_weights, single_gpu  # noqa: E402
from velvetoptimizer_b200 import MoEConfig  # noqa: E402
from velvetoptimizer_b200.ep import ExpertParallelMoE  # noqa: E402

PEER_TIMEOUT = 0x105  # device status: a wait on a peer's flag gave up


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    from datetime import timedelta
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    failures = []
    try:
        cfg = MoEConfig(hidden_size=256, intermediate_size=256, moe_num_experts=2 * world,
                        moe_top_k=2)
        T = 256
        w = global_weights(cfg, dev, torch.bfloat16, seed=3)
        g = torch.Generator(device=dev)
        g.manual_seed(50 + rank)
        x = torch.randn(T, cfg.hidden_size, generator=g, device=dev).to(torch.bfloat16)
        layer = ExpertParallelMoE(cfg, w, dev, torch.bfloat16, transport="p2p", max_tokens=T,
                                  chunks=1)
        out, _ = layer(x)
        torch.cuda.synchronize()
        if layer.device_status() != 0:
            failures.append(f"rank {rank}: healthy forward reported a device error")
        dist.barrier()
        if rank == 0:
            t0 = time.time()
            layer(x)                      # rank 1 never joins this forward
            torch.cuda.synchronize()
            took = time.time() - t0
            status = layer.device_status()
            if status != PEER_TIMEOUT:
                failures.append(f"rank 0: expected peer-timeout status 0x{PEER_TIMEOUT:x}, got 0x{status:x}")
            if not 1.0 < took < 60.0:
                failures.append(f"rank 0: the abandoned forward took {took:.1f} s")
            ref, _ = single_gpu(cfg, w, x, torch.bfloat16)  # the context still works
            if not torch.equal(ref, out):
                failures.append("rank 0: single-GPU forward after the timeout differs")
            print(f"rank 0: abandoned forward ended after {took:.1f} s with status 0x{status:x}",
                  flush=True)
        dist.barrier()                    # rank 1 waits here, on the host, launching nothing
        layer.close()
    finally:
        dist.destroy_process_group()
    if failures:
        print("\n".join(failures), flush=True)
        return 1
    print(f"FAULT_OK rank {rank}", flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
