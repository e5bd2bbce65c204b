"""Worker of the two-GPU slab test: one rank per GPU over NCCL (launched by torch.distributed.run).

Every rank builds the same SpectralConv and input, runs its slab through SlabSpectralConv (CUDA
stages + two NCCL all-to-alls), the slabs are gathered and rank 0 writes the relative L2 error
against the single-GPU forward to the JSON file named on the command line.  The same for a whole 3D
FNO through SlabFNO (lifting with the slab's grid offset, chain kernels on the local planes, every
spectral layer slab-decomposed).
"""

import datetime
import json
import os
import sys

import torch
import torch.distributed as dist

import neuraloperator_b200 as nb
from neuraloperator_b200.distributed import SlabFNO, SlabSpectralConv


def main(out_path):
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(int(os.environ["LOCAL_RANK"]))
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    try:
        torch.manual_seed(0)
        conv = nb.SpectralConv(3, 2, (32, 32, 32)).cuda()
        g = torch.Generator(device="cpu").manual_seed(1)
        with torch.no_grad():
            w = conv.weight.tensor
            w.copy_(torch.complex(torch.randn(w.shape, generator=g), torch.randn(w.shape, generator=g)).cuda() * 0.05)
        x = torch.randn((1, 3, 256, 256, 256), generator=g).cuda()
        nx = 256 // world
        with torch.no_grad():
            y_slab = SlabSpectralConv(conv)(x[:, :, rank * nx:(rank + 1) * nx].contiguous())
            parts = [torch.empty_like(y_slab) for _ in range(world)]
            dist.all_gather(parts, y_slab)
            err = None
            if rank == 0:
                y = torch.cat(parts, dim=2)
                ref = conv(x)
                err = ((y - ref).norm() / ref.norm()).item()
            # the whole FNO on the slabs
            torch.manual_seed(2)
            model = nb.FNO(n_modes=(32, 32, 32), in_channels=3, out_channels=3, hidden_channels=8,
                           n_layers=4).cuda().eval()
            xm = torch.randn((1, 3, 256, 256, 256), generator=g).cuda()
            out_slab = SlabFNO(model)(xm[:, :, rank * nx:(rank + 1) * nx].contiguous())
            parts = [torch.empty_like(out_slab) for _ in range(world)]
            dist.all_gather(parts, out_slab)
            if rank == 0:
                out = torch.cat(parts, dim=2)
                ref = model(xm)
                err_fno = ((out - ref).norm() / ref.norm()).item()
                with open(out_path, "w") as f:
                    json.dump({"err": err, "err_fno": err_fno, "world": world}, f)
        torch.cuda.synchronize()
        dist.barrier()
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main(sys.argv[1])
