"""Worker of tests/test_gpu_ep.py::test_ep_nccl_matches_single_gpu, one process per GPU
under torchrun: expert-parallel decode over NCCL, compared on rank 0 with the
single-GPU batched path holding all experts.  Exit status 0 = bit-identical."""
from __future__ import annotations

import os
import sys
from datetime import timedelta
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))


def main() -> int:
    import torch
    import torch.distributed as dist
    from tinygiant_b200.engine import MoEModel
    from tinygiant_b200.ep import EPMoEModel
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120))
    H, I, E, K, L, T = 2048, 768, 128, 8, 3, int(os.environ.get("EP_TOKENS", "5"))
    ok = True
    try:
        ep = EPMoEModel(H, I, E, K, L, rank=rank, size=world, device=local)
        ep.fill_synthetic(2024)
        p2p = os.environ.get("EP_P2P", "0") == "1"
        if p2p:
            ep.enable_p2p(64)
        g = torch.Generator(device="cuda").manual_seed(99)
        X = torch.randn(T, H, generator=g, device="cuda")           # the same tokens on every rank
        X0 = X.clone()
        ep.decode(X)
        torch.cuda.synchronize()
        if p2p:
            ep.p2p_status()
        same = torch.tensor([1.0], device="cuda")
        if rank == 0:
            full = MoEModel(H, I, E, K, L, device=local)
            full.fill_synthetic(2024)
            full.decode_batched(X0)
            torch.cuda.synchronize()
            ok = torch.equal(X.view(torch.int32), X0.view(torch.int32))
            full.close()
            same[0] = 1.0 if ok else 0.0
        dist.broadcast(same, 0)                                        # every rank takes the same steps
        ok = bool(same.item() == 1.0)
        ep.close()                                                     # disconnect, barrier, free
    finally:
        dist.destroy_process_group()
    if rank == 0:
        print("ep-p2p" if os.environ.get("EP_P2P") == "1" else "ep-nccl", "bit-identical" if ok else "MISMATCH",
              flush=True)
    return 0 if ok else 1


if __name__ == "__main__":
    sys.exit(main())
