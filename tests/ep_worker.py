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
    H, I, E, K, T = 2048, 768, 128, 8, int(os.environ.get("EP_TOKENS", "5"))
    # an odd layer count and several decodes back to back: consecutive exchange calls must
    # alternate receive buffers across decode boundaries too
    L, R = int(os.environ.get("EP_LAYERS", "3")), int(os.environ.get("EP_REPEAT", "1"))
    ok = True
    try:
        ep = EPMoEModel(H, I, E, K, L, rank=rank, size=world, device=local)
        ep.fill_synthetic(2024)
        p2p = os.environ.get("EP_P2P", "0") == "1"
        if p2p:
            ep.enable_p2p(64)
        full = None
        if rank == 0:
            full = MoEModel(H, I, E, K, L, device=local)
            full.fill_synthetic(2024)
        same = torch.tensor([1.0], device="cuda")
        for rep in range(R):
            g = torch.Generator(device="cuda").manual_seed(99 + rep)
            X = torch.randn(T, H, generator=g, device="cuda")       # the same tokens on every rank
            X0 = X.clone()
            ep.decode(X)
            torch.cuda.synchronize()
            if p2p:
                ep.p2p_status()
            if rank == 0:
                full.decode_batched(X0)
                torch.cuda.synchronize()
                if not torch.equal(X.view(torch.int32), X0.view(torch.int32)):
                    same[0] = 0.0
        if full is not None:
            full.close()
        if p2p and os.environ.get("EP_SKIP") == "1":
            # rank 1 skips one exchange: rank 0's combine waits for a flag that never comes,
            # gives up at the wait limit (~1 s) and reports it; nothing faults.  Rank 1 has
            # no kernel in flight meanwhile, and both meet again in close().
            from tinygiant_b200._lib import TG_ETIMEOUT, TinyGiantError
            if rank == 0:
                Xs = torch.randn(T, H, device="cuda")
                ep.moe_layer(0, Xs)
                torch.cuda.synchronize()
                try:
                    ep.p2p_status()
                    same[0] = 0.0                                      # the wait should have run out
                except TinyGiantError as err:
                    if err.code != TG_ETIMEOUT:
                        same[0] = 0.0
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
