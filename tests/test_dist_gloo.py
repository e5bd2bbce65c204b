"""Multi-process host logic on CPU (gloo, world size 2): batch sharding and the 3D slab exchange.

The slab test runs ``SlabSpectralConv`` with its three compute stages replaced by a host emulation
that produces / consumes the same buffer layouts as the CUDA stages:
  send1 = [plane block][b, c, local x][8]          (forward planes)
  recv1 = [source rank][my block][b, c][source x][8]
  send2 = [destination rank][my block][b, o][destination x][8]
  recv2 = [plane block][b, o, local x][8]            (inverse planes)
so the exchange logic (split rule, byte counts, segment order, weight-block mapping) is checked
end to end against the oracle, including an uneven block split.
"""

import math
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import neuraloperator_b200 as nb
import oracle
from neuraloperator_b200.distributed import SlabSpectralConv, gather_batch, shard_batch


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _c64(t):
    return t.view(torch.complex64)


def _u8(t):
    return t.contiguous().view(torch.uint8).reshape(-1)


class EmulatedSlab(SlabSpectralConv):
    """Host emulation of the three libnop_b200 slab stages (same layouts, plain torch on CPU)."""

    def _geo(self, x_slab, world):
        return self.conv.geometry([x_slab.shape[2] * world, *x_slab.shape[3:]])

    def stage_planes_fwd(self, x_slab, lay):
        geo = self._geo(x_slab, lay.world)
        B, C, nx, Ny, Nz = x_slab.shape
        MX, MY, KZ = geo.kept
        spec = torch.fft.rfft2(x_slab.double(), dim=(-2, -1)) * geo.fwd_scale      # [B, C, nx, Ny, Nz/2+1]
        uy = [(m - geo.fwd_off[1]) % Ny for m in range(MY)]
        kept = spec[..., uy, :KZ].reshape(B * C * nx, MY * KZ)                       # plane modes m_p
        blocks = kept.reshape(B * C * nx, lay.blocks, 8).permute(1, 0, 2)           # [Qp][L][8]
        return _u8(blocks.to(torch.complex64))

    def stage_modes(self, recv1, x_slab, lay):
        geo = self._geo(x_slab, lay.world)
        B, Ci, nx = x_slab.shape[:3]
        Co = self.conv.out_channels
        MX, MY, KZ = geo.kept
        Nx = nx * lay.world
        qc, qb = lay.block_count(lay.rank), lay.block_begin(lay.rank)
        r1 = _c64(recv1).reshape(lay.world, qc, B * Ci, nx, 8).to(torch.complex128)
        lines = r1.permute(1, 2, 0, 3, 4).reshape(qc, B * Ci, Nx, 8)                 # x lines per (block, bc, j)
        ux = torch.tensor([(m - geo.fwd_off[0]) % Nx for m in range(MX)])
        xs = torch.fft.fft(lines, dim=2)[:, :, ux, :]                                 # [qc, BCi, MX, 8]
        w = self.conv.weight.tensor.detach().reshape(Ci, Co, MX, MY * KZ).to(torch.complex128)
        modes = (qb + torch.arange(qc))[:, None] * 8 + torch.arange(8)[None, :]      # plane mode of (block, j)
        wsel = w[:, :, :, modes]                                                      # [Ci, Co, MX, qc, 8]
        xsb = xs.reshape(qc, B, Ci, MX, 8)
        ys = torch.einsum("qbimj,iomqj->qbomj", xsb, wsel).reshape(qc, B * Co, MX, 8)
        ui = torch.tensor([(m - geo.inv_off[0]) % Nx for m in range(MX)])
        xg = torch.arange(Nx)
        basis = torch.exp(2j * math.pi * torch.outer(ui, xg).double() / Nx)           # [MX, Nx]
        full = torch.einsum("qcmj,mx->qcxj", ys, basis)                               # [qc, BCo, Nx, 8]
        send2 = full.reshape(qc, B * Co, lay.world, nx, 8).permute(2, 0, 1, 3, 4)     # [dest][qc][BCo][nx][8]
        return _u8(send2.to(torch.complex64))

    def stage_planes_inv(self, recv2, x_slab, lay, addend=None, apply_gelu=False, out=None):
        geo = self._geo(x_slab, lay.world)
        B, _, nx, Ny, Nz = x_slab.shape
        Co = self.conv.out_channels
        MX, MY, KZ = geo.kept
        r2 = _c64(recv2).reshape(lay.blocks, B * Co * nx, 8).permute(1, 0, 2).reshape(B, Co, nx, MY, KZ)
        full = torch.zeros(B, Co, nx, Ny, Nz // 2 + 1, dtype=torch.complex128)
        uy = [(m - geo.inv_off[1]) % Ny for m in range(MY)]
        full[..., uy, :KZ] = r2.to(torch.complex128)
        full = torch.fft.ifft(full, dim=-2, norm="forward")
        full[..., 0] = full[..., 0].real.to(full.dtype)
        y = torch.fft.irfft(full, n=Nz, dim=-1, norm="forward") * geo.inv_scale
        y = (y + self.conv.bias.detach().double()).float()
        if out is not None:
            out.copy_(y)
            return out
        return y


def _slab_worker(rank, world, port, result):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        torch.manual_seed(0)
        n, modes = (8, 16, 16), (8, 8, 8)      # kept (8, 8, 5): 40 plane modes = 5 blocks -> split 3 / 2
        conv = nb.SpectralConv(3, 2, modes)
        g = torch.Generator().manual_seed(1)
        with torch.no_grad():
            conv.weight.tensor.copy_(torch.complex(torch.randn(conv.weight.shape, generator=g),
                                                   torch.randn(conv.weight.shape, generator=g)) * 0.3)
        x = torch.randn((2, 3, *n), generator=g)
        nx = n[0] // world
        y_slab = EmulatedSlab(conv)(x[:, :, rank * nx:(rank + 1) * nx])
        parts = [torch.empty_like(y_slab) for _ in range(world)]
        dist.all_gather(parts, y_slab)
        if rank == 0:
            y = torch.cat(parts, dim=2)
            ref = oracle.spectral_conv(x, conv.weight.tensor.detach(), conv.bias.detach(), modes)
            result["err"] = ((y - ref).norm() / ref.norm()).item()
            lay = EmulatedSlab(conv).layout(x[:, :, :nx])
            result["splits"] = (lay.block_count(0), lay.block_count(1))
        # batch sharding round trip
        xb = torch.arange(8.0).reshape(4, 2)
        back = gather_batch(shard_batch(xb, rank, world))
        if rank == 0:
            result["batch_ok"] = bool(torch.equal(back, xb))
    finally:
        dist.destroy_process_group()


def test_slab_exchange_and_batch_sharding_gloo():
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        result = mgr.dict()
        mp.start_processes(_slab_worker, args=(2, _free_port(), result), nprocs=2, start_method="spawn", join=True)
        assert result["splits"] == (3, 2)
        assert result["batch_ok"]
        assert result["err"] <= 1e-5, result["err"]
