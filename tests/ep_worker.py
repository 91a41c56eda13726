"""Worker of tests/test_gpu_ep.py::test_ep_multi_gpu_matches_single_gpu, one process per
GPU under torchrun: expert-parallel decode compared on rank 0 with one GPU holding all
experts.  EP_MODE:
  nccl   per layer: partial step, NCCL all-reduce, combine (T tokens at once), against
         the single-GPU batched path
  p2p    the same with the NVLink push exchange instead of the all-reduce
  fused  one persistent kernel per rank and token over all layers (tgx_ep_decode_step),
         against the single-GPU fused step (tgx_decode_step); every rank's hidden
         state must equal rank 0's
  dispatch  every rank holds its own share of the T tokens; each (token, slot) pair
         travels to its expert's holder and back (NCCL all-to-alls, tgx_ep_dispatch*),
         against the single-GPU batched path
  dispatch_p2p  the same through the ranks' IPC regions over NVLink, no host sync
         (tgx_ep_dispatch_p2p_*)
EP_SKIP=1 afterwards makes rank 1 skip one step: rank 0's bounded wait must run out and
report TG_ETIMEOUT, nothing faults, and (fused) both ranks recover and decode bit-exact
again.  Exit status 0 = bit-identical."""
from __future__ import annotations

import os
import sys
from datetime import timedelta
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))


def main() -> int:
    import torch
    import torch.distributed as dist
    from tinygiant_b200._lib import TG_ETIMEOUT, TinyGiantError
    from tinygiant_b200.engine import MoEModel
    from tinygiant_b200.ep import EPMoEModel
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120))
    mode = os.environ.get("EP_MODE", "nccl")
    H, I, E, K, T = 2048, 768, 128, 8, int(os.environ.get("EP_TOKENS", "5"))
    # odd layer counts and several decodes back to back: consecutive exchange calls (and
    # fused steps) must alternate receive buffers across decode boundaries too
    L, R = int(os.environ.get("EP_LAYERS", "3")), int(os.environ.get("EP_REPEAT", "1"))
    ok = True
    try:
        ep = EPMoEModel(H, I, E, K, L, rank=rank, size=world, device=local)
        ep.fill_synthetic(2024)
        if mode == "p2p":
            ep.enable_p2p(64)
        elif mode == "fused":
            ep.enable_fused()
        elif mode == "dispatch_p2p":
            ep.enable_dispatch_p2p(-(-T // world))
        full = None
        if rank == 0:
            full = MoEModel(H, I, E, K, L, device=local)
            full.fill_synthetic(2024)
        same = torch.tensor([1.0], device="cuda")

        def fused_tokens(X):
            for t in range(X.shape[0]):
                ep.decode_step(X[t])
            ep.fused_status()

        def check_against_full(X, X0):
            # every rank holds the same state; rank 0's equals one GPU's
            xs = [torch.empty_like(X) for _ in range(world)]
            dist.all_gather(xs, X)
            if mode.startswith("dispatch"):   # X: every rank's share, gathered back into the T tokens
                xs = [X]
            if rank == 0:
                if mode == "fused":
                    for t in range(X0.shape[0]):
                        full.decode_step(X0[t], eager=True)
                else:
                    full.decode_batched(X0)
                torch.cuda.synchronize()
                for x in xs + [X]:
                    if not torch.equal(x.view(torch.int32), X0.view(torch.int32)):
                        same[0] = 0.0

        for rep in range(R):
            g = torch.Generator(device="cuda").manual_seed(99 + rep)
            X = torch.randn(T, H, generator=g, device="cuda")       # the same tokens on every rank
            X0 = X.clone()
            dist.barrier()      # the ranks' steps start together (a lagging rank would be waited on)
            if mode == "fused":
                fused_tokens(X)
            elif mode.startswith("dispatch"):
                sizes = [len(c) for c in torch.tensor_split(torch.arange(T), world)]
                mine = torch.tensor_split(X, world)[rank].contiguous()
                if mode == "dispatch":
                    ep.decode_dispatch(mine)
                else:
                    ep.decode_dispatch_p2p(mine)
                    ep.dispatch_p2p_status()
                ep.status()
                pad = torch.zeros(max(sizes), H, device="cuda")
                pad[: sizes[rank]] = mine
                parts = [torch.empty_like(pad) for _ in range(world)]
                dist.all_gather(parts, pad)
                X = torch.cat([p[:n] for p, n in zip(parts, sizes)])
            else:
                ep.decode(X)
                torch.cuda.synchronize()
                if mode == "p2p":
                    ep.p2p_status()
            check_against_full(X, X0)
        if mode in ("p2p", "fused", "dispatch_p2p") and os.environ.get("EP_SKIP") == "1":
            # rank 1 skips a step: rank 0 waits for down values (p2p: an epoch flag) that
            # never come, gives up at the wait limit and reports it; nothing faults.  Rank 1
            # has no kernel in flight meanwhile.
            dist.barrier()
            if mode == "fused":
                ep.set_wait_limit(4_000_000)                           # ~2 ms
            if rank == 0:
                Xs = torch.randn(T, H, device="cuda")
                try:
                    if mode == "fused":
                        ep.decode_step(Xs[0])
                        ep.fused_status()
                    elif mode == "dispatch_p2p":
                        ep.moe_layer_dispatch_p2p(0, Xs[:1].contiguous())
                        ep.dispatch_p2p_status()
                    else:
                        ep.moe_layer(0, Xs)
                        torch.cuda.synchronize()
                        ep.p2p_status()
                    same[0] = 0.0                                      # the wait should have run out
                except TinyGiantError as err:
                    if err.code != TG_ETIMEOUT:
                        same[0] = 0.0
            if mode == "fused":
                # every rank restarts its launch count above every rank's, then decodes again
                ep.fused_recover()
                ep.set_wait_limit(0)
                g = torch.Generator(device="cuda").manual_seed(7)
                X = torch.randn(2, H, generator=g, device="cuda")
                X0 = X.clone()
                dist.barrier()
                fused_tokens(X)
                check_against_full(X, X0)
        if full is not None:
            full.close()
        dist.broadcast(same, 0)                                        # every rank takes the same steps
        ok = bool(same.item() == 1.0)
        ep.close()                                                     # disconnect, barrier, free
    finally:
        dist.destroy_process_group()
    if rank == 0:
        print("ep-" + mode, "bit-identical" if ok else "MISMATCH", flush=True)
    return 0 if ok else 1


if __name__ == "__main__":
    sys.exit(main())
