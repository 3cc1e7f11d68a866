"""MailboxAR in a few lines, one process per device:

    torchrun --nproc-per-node 2 --master-addr 127.0.0.1 examples/allreduce_demo.py            # GPUs (NCCL group)
    torchrun --nproc-per-node 2 --master-addr 127.0.0.1 examples/allreduce_demo.py --cpu      # CPU transport (gloo)

Allreduces a rank-valued tensor in-house (falling back to the process group
above the size limit), checks the sum, captures one call in a CUDA graph on
GPUs, and prints the communicator's ready state and per-path counters.
"""
import argparse
import importlib
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
par = importlib.import_module("3080_mod_p2p_sglang_patch_b200.parallel")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--cpu", action="store_true", help="CPU transport over gloo (no GPU needed)")
    ap.add_argument("--numel", type=int, default=1 << 20)
    args = ap.parse_args()
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    if args.cpu:
        dist.init_process_group("gloo")
        device = torch.device("cpu")
    else:
        local = int(os.environ.get("LOCAL_RANK", rank))
        torch.cuda.set_device(local)
        device = torch.device("cuda", local)
        dist.init_process_group("nccl", device_id=device)
    ar = par.MailboxAR(None, device)
    x = torch.full((args.numel,), float(rank + 1), dtype=torch.bfloat16, device=device)
    y = ar.all_reduce(x)  # in-house when the communicator is up and the size fits, else the process group
    want = world * (world + 1) / 2
    assert bool(torch.all(y.float() == want)), "wrong sum"
    if not args.cpu and not ar.disabled:
        g = torch.cuda.CUDAGraph()
        with ar.capture():  # nothing to register: buffers never move
            with torch.cuda.graph(g):
                yg = ar.custom_all_reduce(x)
        x.fill_(2.0)
        g.replay()
        torch.cuda.synchronize()
        assert bool(torch.all(yg.float() == 2.0 * world)), "wrong sum after replay"
    if rank == 0:
        print({"transport": getattr(ar, "transport", None), "disabled": ar.disabled, "err": ar.err(),
               "counters": {k: v for k, v in ar.counters.items() if v}})
    ar.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
