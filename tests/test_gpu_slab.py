"""3D slab decomposition on the GPU.

* The C ABI's split (nop_spectral_slab_info) equals the host rule (SlabLayout).
* Several ranks emulated on ONE GPU: every rank's three CUDA stages run in one process and the two
  all-to-alls are done by copying the per-peer segments, so the segmented layouts are checked on a
  single B200 (world 2 and 4, uneven block splits, fused epilogue).
* Two real ranks over NCCL (skipped with fewer than two GPUs): ``slab_nccl_worker.py`` under
  torch.distributed.run, compared with the single-GPU forward.
Tolerance: relative L2 <= 1e-5 (fp32 contraction) against the single-GPU fused path, which the
parity tests pin to the oracle.
"""

import json
import os
import subprocess
import sys

import pytest
import torch

import neuraloperator_b200 as nb
from conftest import ROOT, rel_l2
from neuraloperator_b200 import _lib, ops
from neuraloperator_b200.distributed import SlabLayout, SlabSpectralConv

pytestmark = pytest.mark.gpu

TOL_FP32 = 1e-5


@pytest.fixture(autouse=True, scope="module")
def _needs_cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")


def _conv(ci, co, modes, seed=0, factorization=None):
    torch.manual_seed(seed)
    kw = {} if factorization is None else dict(factorization=factorization, rank=0.5)
    conv = nb.SpectralConv(ci, co, modes, **kw).cuda()
    if factorization is None:
        with torch.no_grad():
            w = conv.weight.tensor
            g = torch.Generator(device="cpu").manual_seed(seed + 1)
            w.copy_(torch.complex(torch.randn(w.shape, generator=g), torch.randn(w.shape, generator=g)).cuda() * 0.05)
            conv.bias.copy_(torch.randn(conv.bias.shape, generator=g).cuda() * 0.1)
    return conv


def run_emulated(slab: SlabSpectralConv, x: torch.Tensor, world: int, addend=None, apply_gelu=False):
    """All ranks of a slab decomposition on one device; the exchanges are segment copies."""
    nx = x.shape[2] // world
    xs = [x[:, :, r * nx:(r + 1) * nx].contiguous() for r in range(world)]
    lays = [slab.layout(xs[r], rank=r, world=world) for r in range(world)]
    send1 = [slab.stage_planes_fwd(xs[r], lays[r]) for r in range(world)]
    seg1 = [list(torch.split(send1[s], lays[s].send1_split())) for s in range(world)]
    recv1 = [torch.cat([seg1[s][r] for s in range(world)]) for r in range(world)]
    for r in range(world):
        assert recv1[r].numel() == sum(lays[r].recv1_split())
    send2 = [slab.stage_modes(recv1[r], xs[r], lays[r]) for r in range(world)]
    seg2 = [list(torch.split(send2[s], lays[s].send2_split())) for s in range(world)]
    recv2 = [torch.cat([seg2[s][r] for s in range(world)]) for r in range(world)]
    ys = []
    for r in range(world):
        a = None if addend is None else addend[:, :, r * nx:(r + 1) * nx]
        ys.append(slab.stage_planes_inv(recv2[r], xs[r], lays[r], addend=a, apply_gelu=apply_gelu))
    return torch.cat(ys, dim=2)


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("modes", [(32, 32, 32), (64, 64, 64)])
def test_slab_info_matches_host_layout(world, modes):
    conv = _conv(3, 5, modes)
    geo = conv.geometry([256, 256, 256])
    desc = ops.make_desc(geo, 2, 3, 5, engine="fast")
    x_slab = torch.empty((2, 3, 256 // world, 256, 256), device="meta")
    for r in range(world):
        plan = _lib.Plan(desc, slab=(r, world))
        info = plan.slab_info
        lay = SlabSpectralConv(conv).layout(x_slab, rank=r, world=world)
        assert (info.rank, info.world, info.x_begin, info.x_count) == (r, world, r * lay.nx, lay.nx)
        assert info.plane_blocks == lay.blocks
        assert [info.block_count[s] for s in range(world)] == [lay.block_count(s) for s in range(world)]
        assert [info.block_begin[s] for s in range(world)] == [lay.block_begin(s) for s in range(world)]
        assert [info.send1_split[s] for s in range(world)] == lay.send1_split()
        assert [info.recv1_split[s] for s in range(world)] == lay.recv1_split()
        assert [info.send2_split[s] for s in range(world)] == lay.send2_split()
        assert [info.recv2_split[s] for s in range(world)] == lay.recv2_split()
        assert info.send1_bytes == sum(lay.send1_split()) and info.recv2_bytes == sum(lay.recv2_split())


@pytest.mark.parametrize("world", [2, 4])
@pytest.mark.parametrize("modes", [(32, 32, 32), (64, 64, 64)])
def test_slab_emulated_ranks_match_single_gpu(world, modes):
    conv = _conv(3, 2, modes)
    g = torch.Generator(device="cpu").manual_seed(7)
    x = torch.randn((1, 3, 256, 256, 256), generator=g).cuda()
    with torch.no_grad():
        ref = conv(x)
        y = run_emulated(SlabSpectralConv(conv), x, world)
    torch.cuda.synchronize()
    assert y.shape == ref.shape
    assert rel_l2(y, ref) <= TOL_FP32


def test_slab_emulated_fused_epilogue():
    conv = _conv(2, 2, (32, 32, 32), seed=3)
    g = torch.Generator(device="cpu").manual_seed(11)
    x = torch.randn((2, 2, 256, 256, 256), generator=g).cuda()
    skip = torch.randn((2, 2, 256, 256, 256), generator=g).cuda()
    with torch.no_grad():
        ref = torch.nn.functional.gelu(conv(x) + skip)
        y = run_emulated(SlabSpectralConv(conv), x, 2, addend=skip, apply_gelu=True)
    assert rel_l2(y, ref) <= TOL_FP32


def test_slab_emulated_tucker():
    conv = _conv(4, 4, (32, 32, 32), seed=5, factorization="tucker")
    g = torch.Generator(device="cpu").manual_seed(13)
    x = torch.randn((1, 4, 256, 256, 256), generator=g).cuda()
    with torch.no_grad():
        ref = conv(x)
        y = run_emulated(SlabSpectralConv(conv), x, 2)
    assert rel_l2(y, ref) <= TOL_FP32


def _free_port() -> int:
    """A TCP port on 127.0.0.1 that nothing listens on right now (the rendezvous port)."""
    import socket
    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_slab_two_gpus_nccl(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    out = tmp_path / "slab.json"
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", PYTHONPATH=ROOT)
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", f"--master-port={_free_port()}",
           os.path.join(ROOT, "tests", "slab_nccl_worker.py"), str(out)]
    subprocess.run(cmd, check=True, timeout=600, env=env, cwd=ROOT)
    res = json.loads(out.read_text())
    assert res["err"] <= TOL_FP32, res
    assert res["err_fno"] <= TOL_FP32, res
