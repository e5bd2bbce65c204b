"""Benchmark of the FNO forward on B200 (driver contract: one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config c5]

Default workload: the whole FNO forward (the headline metric, "FNO fwd samples/s") on the largest
configuration that fits one GPU, configs[4]: FNO 3D, 256^3 grid, batch 8, hidden 32, n_modes (32, 32, 32),
3 input (+3 grid) and 3 output channels, fp32.  Input: three seeded periodic Gaussian random fields
with covariance (-Lap + 16 I)^-2 (no dataset); weights: the reference initialisers, seed 0.
A step is one forward over the batch.  N = 1: the batch on one GPU.  N > 1 (torchrun): the 256^3 grid
is slab-decomposed along x across the ranks, with NCCL all-to-alls of the kept modes inside every
spectral layer (strong scaling: the global batch stays 8); the job value is 8 / max-over-ranks(time).

* value        : samples/s with the input resident in HBM (CUDA events on the launching stream).
* e2e          : the same through FNO.forward_host / SlabFNO.forward_host -- pinned host input in,
                 pinned host output out, every copy inside the timed region.
* roofline     : the forward's dominant kernel (most time per forward): its compulsory bytes per
                 launch over its mean launch time from CUDA events recorded between the launches of
                 one instrumented forward, against the measured HBM copy bandwidth; kernels[] lists all.
* cpu_baseline : the oracle (the reference's torch CPU path restated in oracle/) on the host cores,
                 one sample's forward.
--impl reference times that CPU path as the reference arm.  --model layer runs the single-SpectralConv
benchmarks (configs[1], the C2 microbench, by default) and their training step (--pass train).
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

E2E_STREAMS = 3
METRIC = "FNO fwd samples/s/GPU at 1–8 B200; spectral block % of HBM/tensor roofline"
HBM_FALLBACK_GBS = 6533.2  # measured copy bandwidth on this pool (MEASURED_PEAKS.json at round start)

# DRAM bytes (read + write) per launch of the dominant kernel, from ncu captures summarised under
# (small-batch capture scaled to the full batch; traffic grows with the number of planes)
TRAFFIC = {
    # `ncu --set full` of the C2 block at batch 8, x 8 (reads + writes during the kernel; the
    # plane kernels' traffic grows with the number of planes)
    ("c2", "plane_inv"): 8 * (8.701952e6 + 79.316992e6),
    ("c2", "plane_fwd"): 8 * (134.246144e6 + 4.028928e6),
    # full-size capture of the C2 contraction (one launch)
    ("c2", "contraction"): 207.854080e6 + 10.398976e6,
    # C5 model at 128^3, batch 1: capture x 64 (the chain's traffic grows with the points)
    ("c5", "chain_block"): 64 * (537.109760e6 + 227.285760e6),
    ("c5", "chain_lifting"): 64 * (25.244928e6 + 209.326080e6),
    ("c5", "chain_last_block_projection"): 64 * (537.034240e6 + 17.639168e6),
}

# name -> (description, batch, Ci, Co, grid, n_modes, factorization)
CONFIGS = {
    "c1": ("darcy2d_layer", 16, 32, 32, (128, 128), (16, 16), None),
    "c2": ("spectralconv2d_micro", 64, 64, 64, (256, 256), (64, 64), None),
    "c3": ("burgers1d_layer", 256, 64, 64, (8192,), (16,), None),
    "c4": ("tfno2d_ns_layer", 32, 64, 64, (512, 512), (64, 64), "tucker"),
    "c5": ("fno3d_layer", 8, 32, 32, (256, 256, 256), (32, 32, 32), None),
}


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured (MEASURED_PEAKS.json)"
    except Exception:  # noqa: BLE001
        return HBM_FALLBACK_GBS, "measured on this pool (recorded value; MEASURED_PEAKS.json absent)"


class ClockSampler:
    """SM clock and clock-event (throttle) reasons sampled through NVML every 2 ms while the timed
    region runs (read-only queries; nothing on the GPU is changed)."""

    REASONS = {  # NVML clocks-event reason bits
        0x8: "hw_slowdown", 0x40: "hw_thermal_slowdown", 0x20: "sw_thermal_slowdown", 0x4: "sw_power_cap",
        0x80: "hw_power_brake_slowdown", 0x2: "applications_clocks_setting",
    }

    def __init__(self, index: int, period_s: float = 0.002):
        self.index = index
        self.period = period_s
        self.samples = []
        self.max_mhz = None
        self._stop = threading.Event()
        self._t = None

    def __enter__(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            vis = os.environ.get("CUDA_VISIBLE_DEVICES")
            phys = int(vis.split(",")[self.index]) if vis else self.index
            self._h = pynvml.nvmlDeviceGetHandleByIndex(phys)
            self._nv = pynvml
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        except Exception:  # noqa: BLE001
            self._t = None
        return self

    def _run(self):
        nv = self._nv
        while not self._stop.is_set():
            try:
                mhz = nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM)
                reasons = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                self.samples.append((mhz, reasons))
            except Exception:  # noqa: BLE001
                pass
            time.sleep(self.period)

    def __exit__(self, *exc):
        self._stop.set()
        if self._t is not None:
            self._t.join(timeout=2)
        return False

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0, "source": "nvml"}
        reasons = set()
        for _, r in self.samples:
            for bit, name in self.REASONS.items():
                if r & bit:
                    reasons.add(name)
        return {"sm_mhz": statistics.median(m for m, _ in self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(reasons), "samples": len(self.samples), "source": "nvml"}


def make_inputs(cfg, device, seed=0):
    """Synthetic input and seeded weights with the config's shapes (no dataset is available)."""
    import neuraloperator_b200 as nb
    desc, batch, ci, co, grid, modes, fact = cfg
    g = torch.Generator(device="cpu").manual_seed(seed)
    kw = {}
    if fact:
        kw = dict(factorization=fact, implementation="factorized", rank=0.1)
    conv = nb.SpectralConv(ci, co, modes, **kw)
    std = math.sqrt(2.0 / (ci + co))
    with torch.no_grad():
        for p in conv.weight.parameters():
            p.copy_(torch.complex(torch.randn(p.shape, generator=g), torch.randn(p.shape, generator=g)) *
                    (std if not fact else 0.5))
        conv.bias.copy_(torch.randn(conv.bias.shape, generator=g) * std)
    conv = conv.to(device)
    x = torch.randn((batch, ci, *grid), generator=g).to(device) if device != "cpu" else \
        torch.randn((batch, ci, *grid), generator=g)
    return conv, x


def bytes_alg(cfg, conv):
    _, batch, ci, co, grid, _, _ = cfg
    p = math.prod(grid)
    w = sum(t.numel() * t.element_size() for t in conv.weight.parameters())
    return batch * ci * p * 4 + batch * co * p * 4 + w + co * 4


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def max_over_ranks(v: float, world: int) -> float:
    if world == 1:
        return v
    import torch.distributed as dist
    t = torch.tensor([v], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world: int):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def capture_graph(fn, stream):
    """One call of `fn` captured into a CUDA graph on a side stream (plans and packed weights exist
    from the warm-up, so capture allocates only workspace from the graph's pool)."""
    try:
        g = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream()
        side.wait_stream(stream)
        with torch.cuda.stream(side), torch.no_grad():
            fn()  # one eager call on the capture stream
            with torch.cuda.graph(g, stream=side):
                fn()
        stream.wait_stream(side)
        torch.cuda.synchronize()
        return g, "cuda_graph"
    except Exception as exc:  # noqa: BLE001
        print(f"graph capture failed, timing eager launches: {exc}", file=sys.stderr)
        torch.cuda.synchronize()
        return None, "eager"


# ---------------------------------------------------------------------------------------------------
# Full FNO / TFNO forward (the headline metric: FNO forward samples/s)
# ---------------------------------------------------------------------------------------------------
# name -> (workload, class, n_modes, hidden, in, out, grid, batch, kwargs, input field)
# The input fields are seeded periodic Gaussian random fields with each benchmark configuration's
# covariance (no dataset is available): (scale, tau^2, alpha) of s^2 (-Lap + tau^2 I)^-alpha,
# plus the Darcy threshold to {3, 12}.
MODELS = {
    "c1": ("fno2d_darcy", "FNO", (16, 16), 32, 1, 1, (128, 128), 16, {}, (1.0, 9.0, 2.0, "darcy")),
    "c3": ("fno1d_burgers", "FNO", (16,), 64, 1, 1, (8192,), 256, {}, (625.0, 25.0, 2.0, None)),
    "c4": ("tfno2d_ns", "TFNO", (64, 64), 64, 1, 1, (512, 512), 32,
           dict(factorization="tucker", implementation="factorized", rank=0.1), (7.0 ** 0.75, 49.0, 2.5, None)),
    "c5": ("fno3d", "FNO", (32, 32, 32), 32, 3, 3, (256, 256, 256), 8, {}, (1.0, 16.0, 2.0, None)),
}


def grf(batch, channels, grid, field, seed, device):
    """Seeded periodic Gaussian random field on [0, 1)^d with covariance s^2 (-Lap + tau^2 I)^-alpha:
    complex white noise times the square root of the covariance's eigenvalues, inverse real FFT (an
    input generator only; the timed path never calls it)."""
    scale, tau2, alpha, kind = field
    gen = torch.Generator(device=device).manual_seed(seed)
    d = len(grid)
    ks = [torch.fft.fftfreq(n, 1.0 / n, device=device) for n in grid[:-1]] + \
         [torch.fft.rfftfreq(grid[-1], 1.0 / grid[-1], device=device)]
    k2 = sum(k.reshape([-1 if i == j else 1 for i in range(d)]) ** 2 for j, k in enumerate(ks))
    sqrt_eig = scale * (4 * math.pi ** 2 * k2 + tau2) ** (-alpha / 2)
    shape = (batch, channels, *k2.shape)
    noise = torch.complex(torch.randn(shape, generator=gen, device=device),
                          torch.randn(shape, generator=gen, device=device)) / math.sqrt(2.0)
    u = torch.fft.irfftn(noise * sqrt_eig, s=list(grid), dim=list(range(2, 2 + d)), norm="forward")
    if kind == "darcy":
        u = torch.where(u >= 0, torch.full_like(u, 12.0), torch.full_like(u, 3.0))
    return u.to(torch.float32).contiguous()


def build_model(cfg_name, device, precision="fp32"):
    import neuraloperator_b200 as nb
    desc, cls, modes, hidden, cin, cout, grid, batch, kw, field = MODELS[cfg_name]
    if precision == "bf16":
        kw = dict(kw, contraction_precision="bf16")
    torch.manual_seed(0)  # random-init weights of the architecture (reference initialisers)
    model = getattr(nb, cls)(n_modes=modes, in_channels=cin, out_channels=cout, hidden_channels=hidden,
                             n_layers=4, **kw)
    return model.to(device).eval()


def oracle_params(model):
    """The model's parameters in the oracle's layout (CPU tensors): fno_forward(x, params, cfg)."""
    lin = lambda fcs: [(fc.weight.detach().cpu(), fc.bias.detach().cpu()) for fc in fcs]  # noqa: E731
    fb = model.fno_blocks
    blocks = []
    kind = "dense"
    for i in range(fb.n_layers):
        w = fb.convs[i].weight
        if hasattr(w, "core"):
            kind = "tucker"
            wp = {"core": w.core.detach().cpu(), "factors": [f.detach().cpu() for f in w.factors]}
        else:
            wp = w.tensor.detach().cpu()
        blocks.append({"weight": wp, "bias": fb.convs[i].bias.detach().cpu(),
                       "fno_skip": fb.fno_skips[i].conv.weight.detach().cpu(), "mlp": lin(fb.channel_mlp[i].fcs),
                       "mlp_skip": fb.channel_mlp_skips[i].weight.detach().cpu()})
    params = {"lifting": lin(model.lifting.fcs), "projection": lin(model.projection.fcs), "blocks": blocks}
    return params, {"n_modes": tuple(model.n_modes), "weight_kind": kind}


def chain_bytes(kind, batch, p, hidden, cin, cout):
    """Compulsory HBM bytes of one chain launch: its inputs and outputs, each touched once."""
    act = batch * hidden * p * 4
    return {"lifting": batch * cin * p * 4 + act, "block": 3 * act,
            "last_block_projection": 2 * act + batch * cout * p * 4, "last_block": 3 * act,
            "projection": act + batch * cout * p * 4}[kind]


class _Marks:
    """CUDA events recorded on the current stream between the launches of one instrumented forward."""

    def __init__(self):
        self.names, self.events = [], []
        self.mark("start")

    def mark(self, name):
        e = torch.cuda.Event(enable_timing=True)
        e.record()
        self.names.append(name)
        self.events.append(e)

    def spans(self):
        return [(self.names[i + 1], self.events[i].elapsed_time(self.events[i + 1]))
                for i in range(len(self.events) - 1)]


def instrumented_forward(model, x, spectral=None, grid_offset=None, grid_sizes=None):
    """The fused forward of FNO.fused_forward launch by launch, with CUDA events between the launches
    (and the library's per-kernel events inside each spectral layer).  Returns (y, [(kernel, ms)],
    [(layer, spectral kernel ms list)])."""
    from neuraloperator_b200 import _lib, pointwise
    plan = model.fused_plan(x, grid_sizes)
    if plan is None:
        raise SystemExit("the model does not take the fused path at this size")
    grid, fuse_proj = plan
    marks = _Marks()
    f1, f2 = model.lifting.fcs
    h = pointwise.chain(x, f1.weight, f1.bias, f2.weight, f2.bias, grid=grid, grid_offset=grid_offset)
    marks.mark("chain_lifting")
    spec = []
    blocks = model.fno_blocks
    last = model.n_layers - 1
    for i in range(model.n_layers):
        conv = blocks.convs[i]
        if spectral is None:
            nk = None
            geo = conv.geometry(list(h.shape[2:]))
            from neuraloperator_b200 import ops
            kind, _, ranks = conv.kernel_operands(geo)
            pl = ops.get_plan(ops.make_desc(geo, h.shape[0], conv.in_channels, conv.out_channels, weight_kind=kind,
                                            ranks=ranks, precision=conv.contraction_precision, engine=conv.engine),
                              h.device.index)
            nk = pl.launches_per_forward
            ev = _lib.LaunchEvents(nk)
            with ev:
                s = conv(h)
            spec.append(ev)
        else:
            s = spectral(i, conv, h)
        marks.mark(f"spectral_{i}")
        mlp, sg = blocks._mlp_parts(i)
        kw = {}
        proj = model.projection if (i == last and fuse_proj) else None
        if proj is not None:
            p1, p2 = proj.fcs
            kw = dict(w3=p1.weight, b3=p1.bias, w4=p2.weight, b4=p2.bias)
        h = pointwise.chain(h, mlp.fcs[0].weight, mlp.fcs[0].bias, mlp.fcs[1].weight, mlp.fcs[1].bias, s=s,
                            w0=blocks.fno_skips[i].conv.weight, act_skip=i != last, act_out=i != last,
                            gate_w=sg.weight if sg is not None else None, gate_b=sg.bias if sg is not None else None,
                            **kw)
        marks.mark(("chain_last_block_projection" if proj is not None else "chain_last_block") if i == last
                   else "chain_block")
    if not fuse_proj:
        p1, p2 = model.projection.fcs
        h = pointwise.chain(h, p1.weight, p1.bias, p2.weight, p2.bias)
        marks.mark("chain_projection")
    torch.cuda.synchronize()
    return h, marks.spans(), [e.durations_ms() for e in spec]


def pin_to_gpu_cpus(local):
    """Restrict this process to the CPUs NVML reports as local to its GPU (its NUMA node), so the pinned
    host buffers allocated next and the copy threads sit on the GPU's side of the socket.  Returns the
    CPU count used, or None when NVML cannot tell."""
    try:
        import pynvml
        props = torch.cuda.get_device_properties(local)
        bus = f"{props.pci_domain_id:08X}:{props.pci_bus_id:02X}:{props.pci_device_id:02X}.0"
        pynvml.nvmlInit()
        h = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
        words = pynvml.nvmlDeviceGetCpuAffinity(h, (os.cpu_count() + 63) // 64)
        cpus = {64 * w + b for w, m in enumerate(words) for b in range(64) if (m >> b) & 1}
        cpus &= os.sched_getaffinity(0)
        if cpus:
            os.sched_setaffinity(0, cpus)
            return len(cpus)
    except Exception:  # noqa: BLE001
        pass
    return None


def copy_ceiling_ms(x_host, y_dev, y_host, steps, world, stream):
    """Per-step time of the e2e path's host traffic alone: x_host -> device and y_dev -> y_host as plain
    cudaMemcpyAsync copies on two streams at once (every rank together), max over ranks."""
    xd = torch.empty(tuple(x_host.shape), dtype=x_host.dtype, device=y_dev.device)
    s_in, s_out = torch.cuda.Stream(y_dev.device), torch.cuda.Stream(y_dev.device)
    torch.cuda.synchronize()
    barrier(world)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(steps):
        s_in.wait_stream(stream)
        s_out.wait_stream(stream)
        with torch.cuda.stream(s_in):
            xd.copy_(x_host, non_blocking=True)
        with torch.cuda.stream(s_out):
            y_host.copy_(y_dev, non_blocking=True)
        stream.wait_stream(s_in)
        stream.wait_stream(s_out)
    b.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    return max_over_ranks(a.elapsed_time(b) / steps, world)


def run_model_train(args, world, rank, local):
    """One FNO / TFNO training step at the configuration's full size: forward, MSE loss against a
    synthetic target, loss.backward() and an Adam step (neuralop/training/trainer.py:629-700 per batch),
    every rank its own batch (weak scaling, gradients not reduced: the data-parallel all-reduce is the
    caller's).  The same step through the module path (torch Conv1d per-pixel layers, NOP_CHAIN=0) is
    timed beside it."""
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    desc, cls, modes, hidden, cin, cout, grid, batch, kw, field = MODELS[args.config]
    if args.batch is not None:
        batch = args.batch
    if args.grid is not None:
        grid = (args.grid,) * len(grid)
        desc += f"_grid{args.grid}"
    model = build_model(args.config, dev, args.precision).train()
    x = grf(batch, cin, grid, field, seed=1 + rank, device=dev)
    target = grf(batch, cout, grid, field, seed=101 + rank, device=dev)
    opt = torch.optim.Adam(model.parameters(), lr=1e-4)
    stream = torch.cuda.current_stream(dev)

    def step():
        opt.zero_grad(set_to_none=True)
        loss = torch.nn.functional.mse_loss(model(x), target)
        loss.backward()
        opt.step()
        return loss

    def timed(steps, warm):
        for _ in range(warm):
            step()
        torch.cuda.synchronize()
        barrier(world)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            loss = step()
        e1.record(stream)
        torch.cuda.synchronize()
        return max_over_ranks(e0.elapsed_time(e1) / steps, world), float(loss)

    fused = model.fused_plan(x) is not None
    with ClockSampler(local) as clocks:
        ms, loss_f = timed(args.steps, args.warmup)
    os.environ["NOP_CHAIN"] = "0"
    try:
        ms_mod, loss_m = timed(max(3, args.steps // 2), 2)
    except torch.OutOfMemoryError:
        ms_mod, loss_m = float("nan"), float("nan")
    finally:
        os.environ.pop("NOP_CHAIN", None)
    if rank != 0:
        return
    line = {
        "metric": "FNO training step (forward + MSE loss + backward + Adam) samples/s", "value": world * batch / (ms / 1e3),
        "unit": "samples/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32" if args.precision == "fp32" else "f32 (bf16 contraction)",
        "data": "synthetic (seeded Gaussian random fields as input and target; no dataset)",
        "config": {"workload": desc + "_train", "model": cls, "global_batch": batch * world, "per_gpu_batch": batch,
                   "grid": list(grid), "hidden_channels": hidden, "n_modes": list(modes), "launch": "eager",
                   "fused_path": fused},
        "module_path": {"samples_per_s": world * batch / (ms_mod / 1e3), "ms_per_step": ms_mod,
                        "definition": "the same step with the per-pixel layers as torch Conv1d (NOP_CHAIN=0)"},
        "loss_fused_vs_module": [loss_f, loss_m],
        "clocks": clocks.summary(),
    }
    print(json.dumps(line), flush=True)


def run_model(args, world, rank, local):
    """FNO / TFNO forward (grid embedding + lifting, 4 FNO blocks, projection) at the configuration's full
    size.  N = 1: the whole batch on one GPU.  N > 1: the 3D configuration is slab-decomposed along x
    (strong scaling: the global batch of 8 is fixed), the 1D / 2D ones shard the batch (weak scaling)."""
    import neuraloperator_b200 as nb  # noqa: F401
    from neuraloperator_b200 import _lib

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if args.config not in MODELS:
        raise SystemExit(f"--model fno: no full-model config named {args.config} (have {sorted(MODELS)})")
    desc, cls, modes, hidden, cin, cout, grid, batch, kw, field = MODELS[args.config]
    if args.batch is not None:
        batch = args.batch
    if args.grid is not None:  # reduced grid for small profiling cases (not a bench number)
        grid = (args.grid,) * len(grid)
        desc += f"_grid{args.grid}"
    slab = world > 1 and len(grid) == 3
    model = build_model(args.config, dev, args.precision)
    gbatch = batch if slab else batch * world
    nx = grid[0] // world if slab else grid[0]
    if slab and grid[0] % world:
        raise SystemExit(f"the slab decomposition needs {grid[0]} x planes to divide by {world} ranks")
    # the synthetic input: every rank draws the same global field (slab) or its own samples (batch shards)
    if slab:
        x_full = grf(batch, cin, grid, field, seed=1, device=dev)
        x = x_full[:, :, rank * nx:(rank + 1) * nx].contiguous()
        del x_full
    else:
        x = grf(batch, cin, grid, field, seed=1 + rank, device=dev)
    runner = None
    if slab:
        from neuraloperator_b200.distributed import SlabFNO
        runner = SlabFNO(model)
        fwd = lambda inp: runner(inp)  # noqa: E731
    else:
        fwd = lambda inp: model(inp)  # noqa: E731
    stream = torch.cuda.current_stream(dev)
    steps, warm = args.steps, args.warmup
    with torch.no_grad():
        if not slab and model.fused_plan(x) is None:
            raise SystemExit("the model does not take the fused path at this size")
        for _ in range(warm):
            y = fwd(x)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        graph, launch = None, "eager"
        if not slab and not args.no_graph:
            barrier(world)
            e0.record(stream)
            y = fwd(x)
            e1.record(stream)
            torch.cuda.synchronize()
            if e0.elapsed_time(e1) < 5.0:  # launch-bound sizes: replay one captured forward
                graph, launch = capture_graph(lambda: fwd(x), stream)
        barrier(world)
        torch.cuda.synchronize()
        with ClockSampler(local) as clocks:
            e0.record(stream)
            for _ in range(steps):
                if graph is not None:
                    graph.replay()
                else:
                    y = fwd(x)
            e1.record(stream)
            torch.cuda.synchronize()
        barrier(world)
        ms = max_over_ranks(e0.elapsed_time(e1) / steps, world)
        del graph

        # ---- one instrumented forward: every launch timed with CUDA events on the launching stream (after
        # one eager forward, so the caching allocator holds every buffer again once the graph is gone) ----
        y = fwd(x)
        torch.cuda.synchronize()
        exch = None
        if slab:
            exch = runner.instrument(True)
            barrier(world)
            y_i, spans, spec_k = instrumented_forward(model, x, spectral=runner.spectral, grid_offset=runner.offset(x),
                                                      grid_sizes=runner.grid_sizes(x))
            exch_ms = [a.elapsed_time(b) for a, b in runner.instrument(False)]
        else:
            y_i, spans, spec_k = instrumented_forward(model, x)
            exch_ms = []
        same = bool(torch.equal(y_i, y))
        del y_i

        # ---- end to end through the public API: pinned host input, pinned host output ----
        ms_e2e, e2e_how, h2d, d2h, ms_copy, numa = float("nan"), None, 0, 0, float("nan"), None
        if not args.no_e2e:
            numa = pin_to_gpu_cpus(local)  # pinned buffers and copy threads on the GPU's own CPUs / node
            x_host = x.cpu().pin_memory()
            y_host = torch.empty(tuple(y.shape), dtype=torch.float32).pin_memory()
            # chunks through the three-stage copy / forward / copy pipeline (only the first chunk's input copy
            # and the last chunk's output copy are not hidden): eight for samples with >= 256 MB of
            # activations (the 3D config), four otherwise, where the forward's host-side launch time per
            # chunk would otherwise exceed its kernels
            per_sample = hidden * math.prod(grid) * 4
            chunk = max(1, batch // (8 if per_sample >= (256 << 20) else 4))
            if slab:  # chunks of two samples: each chunk's spectral layers overlap their own two exchanges
                chunk = 2 if batch % 2 == 0 else 1
            host_call = (lambda: runner.forward_host(x_host, out=y_host, chunk=chunk, synchronize=False)) if slab else \
                (lambda: model.forward_host(x_host, out=y_host, chunk=chunk, n_streams=2, synchronize=False))
            host_call()
            torch.cuda.synchronize()
            ok_e2e = bool(torch.equal(y_host, y.cpu()))
            e2e_steps = max(1, min(steps, 5))
            barrier(world)
            torch.cuda.synchronize()
            f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            f0.record(stream)
            for _ in range(e2e_steps):
                host_call()
            f1.record(stream)
            torch.cuda.synchronize()
            barrier(world)
            ms_e2e = max_over_ranks(f0.elapsed_time(f1) / e2e_steps, world)
            h2d, d2h = x_host.numel() * 4, y_host.numel() * 4
            ms_copy = copy_ceiling_ms(x_host, y, y_host, e2e_steps, world, stream)
            e2e_how = (f"{'SlabFNO' if slab else cls}.forward_host: {batch // chunk} chunks of {chunk} sample(s), "
                       f"H2D / forward / D2H pipelined on three streams, pinned host buffers; output equal to the "
                       f"device forward: {ok_e2e}")

        # ---- slab: rank 0 checks its planes against a single-GPU forward of the whole input ----
        check = None
        if slab and args.slab_check:
            barrier(world)
            if rank == 0:
                x_full = grf(batch, cin, grid, field, seed=1, device=dev)
                y_full = model(x_full)
                ref = y_full[:, :, :nx]
                check = float((y - ref).double().norm() / ref.double().norm())
                del x_full, y_full, ref
            barrier(world)
    if rank != 0:
        return
    hbm, peak_src = peaks()
    p = math.prod(grid) // (world if slab else 1)
    nk = len(spec_k[0]) if spec_k else 0
    kernels = {}

    def add(name, ms_, by):
        k = kernels.setdefault(name, {"name": name, "launches": 0, "ms_total": 0.0, "bytes_alg_per_launch": by})
        k["launches"] += 1
        k["ms_total"] += ms_

    first_conv = model.fno_blocks.convs[0]
    for name, t in spans:
        if name.startswith("chain_"):
            kind = name[len("chain_"):]
            add(name, t, chain_bytes(kind, batch, p, hidden, cin, cout))
        elif not slab:
            pass  # split below from the library's per-kernel events
        else:
            add("spectral_slab_layer", t, None)
    if not slab:
        cfg_l = (desc, batch, hidden, hidden, grid, modes, kw.get("factorization"))
        names = kernel_names_for(first_conv, cfg_l)
        for per in spec_k:
            for n_, t in zip(names, per):
                add(n_, t, kernel_bytes(n_, cfg_l, first_conv))
    klist = []
    for k in kernels.values():
        k["ms"] = k["ms_total"] / k["launches"]
        by = k["bytes_alg_per_launch"]
        k["gbs"] = by / (k["ms"] / 1e3) / 1e9 if by else None
        k["frac"] = k["gbs"] / hbm if by else None
        k["share"] = k["ms_total"] / sum(v["ms_total"] for v in kernels.values())
        klist.append(k)
    dom = max((k for k in klist if k["bytes_alg_per_launch"]), key=lambda k: k["ms_total"])
    total_alg = sum(k["bytes_alg_per_launch"] * k["launches"] for k in klist if k["bytes_alg_per_launch"])
    launches = sum(k["launches"] for k in klist if not k["name"].startswith("spectral_slab"))
    if slab:  # the slab layers' own kernels (their all-to-alls are NCCL's)
        launches += sum(sl.launches(x) for sl in runner.slabs)
    line = {
        "metric": METRIC, "value": gbatch / (ms / 1e3), "unit": "samples/s", "n_gpus": world, "steps": steps,
        "warmup": warm, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong" if slab else "weak",
        "vs_baseline": None, "dtype": "f32" if args.precision == "fp32" else "f32 (bf16 contraction)",
        "data": "synthetic: seeded periodic Gaussian random fields with the configuration's covariance; "
                "seeded random-init weights (no dataset)",
        "config": {"workload": f"{desc}_forward", "model": cls, "global_batch": gbatch,
                   "per_gpu_batch": batch, "grid": list(grid), "hidden_channels": hidden, "n_modes": list(modes),
                   "n_layers": model.n_layers, "in_channels": cin, "out_channels": cout,
                   "parallelism": (f"slab{world}" if slab else f"dp{world}") if world > 1 else "single",
                   "x_planes_per_gpu": nx if slab else None, "launch": launch,
                   "l2": f"activations {batch * hidden * p * 4 / 1e9:.2f} GB > 126 MB L2 (no flush needed)",
                   **{k: v for k, v in kw.items()}},
        "roofline": {"bound": "hbm", "achieved": dom["gbs"], "peak": hbm, "unit": "GB/s", "frac": dom["frac"],
                     "traffic": TRAFFIC.get((args.config, dom["name"])), "kernel": dom["name"],
                     "bytes_alg_per_launch": dom["bytes_alg_per_launch"], "ms_per_launch": dom["ms"],
                     "peak_source": peak_src + " (copy bandwidth, burst)"},
        "model_roofline": {"bound": "hbm", "achieved": total_alg / (sum(k["ms_total"] for k in klist) / 1e3) / 1e9,
                           "peak": hbm, "unit": "GB/s",
                           "frac": total_alg / (sum(k["ms_total"] for k in klist) / 1e3) / 1e9 / hbm,
                           "bytes_alg_per_forward": total_alg,
                           "definition": "sum over the forward's launches of their compulsory bytes (inputs and "
                                         "outputs once each) over the instrumented forward's time"},
        "kernels": klist,
        "instrumented_forward_matches_timed": same,
        "e2e": ({"value": gbatch / (ms_e2e / 1e3), "unit": "samples/s", "h2d_bytes_per_step": h2d,
                 "d2h_bytes_per_step": d2h, "path": e2e_how,
                 "copy_only": gbatch / (ms_copy / 1e3),
                 "ceiling": min(gbatch / (ms_copy / 1e3), gbatch / (ms / 1e3)),
                 "frac_of_ceiling": (gbatch / (ms_e2e / 1e3)) / min(gbatch / (ms_copy / 1e3), gbatch / (ms / 1e3)),
                 "host_cpus": numa,
                 "definition": "ceiling = min(device-resident forward, the same H2D and D2H bytes moved alone "
                               "by cudaMemcpyAsync on two streams at once, every rank together, max over ranks)"}
                if not args.no_e2e else None),
        "gpu_launches": launches * steps,
        "clocks": clocks.summary(),
    }
    if slab:
        lay = runner.slabs[0].layout(x, rank=0, world=world)
        counts = [lay.block_count(r) for r in range(world)]
        line["slab"] = {"exchange_ms_per_layer": [exch_ms[2 * i:2 * i + 2] for i in range(len(exch_ms) // 2)],
                        "exchange_bytes_per_gpu_per_layer": int(sum(lay.send1_split()) + sum(lay.send2_split())),
                        "block_count_per_rank": counts,
                        "block_imbalance": max(counts) / (sum(counts) / len(counts)),
                        "rel_l2_rank0_vs_single_gpu": check}
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline_model(args.config, model)
    print(json.dumps(line), flush=True)


def run_slab(args, cfg, world, rank, local):
    """3D config with the first spatial axis split across the ranks (SlabSpectralConv: local plane
    transforms, NCCL all-to-all of the kept plane modes, x transforms + contraction, all-to-all back,
    local inverse planes).  Every rank holds Nx / world planes of the whole batch: the total work is
    fixed as ranks are added (strong scaling)."""
    import torch.distributed as dist
    from neuraloperator_b200.distributed import SlabSpectralConv

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    desc, batch, ci, co, grid, modes, fact = cfg
    if len(grid) != 3 or grid[0] % world or world < 2:
        raise SystemExit("--parallel slab needs >= 2 ranks and a 3D config whose first axis divides by them")
    conv, _ = make_inputs((desc, 1, ci, co, (1, 1, 1), modes, fact), "cpu", seed=0)  # seeded weights
    conv = conv.to(dev)
    nx = grid[0] // world
    gen = torch.Generator(device=dev).manual_seed(1000 + rank)  # this rank's planes of a synthetic input
    x = torch.randn((batch, ci, nx, *grid[1:]), generator=gen, device=dev)
    slab = SlabSpectralConv(conv)
    stream = torch.cuda.current_stream(dev)
    steps, warm = args.steps, args.warmup
    with torch.no_grad():
        for _ in range(warm):
            y = slab(x)
        torch.cuda.synchronize()
        barrier(world)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(local) as clocks:
            e0.record(stream)
            for _ in range(steps):
                y = slab(x)
            e1.record(stream)
            torch.cuda.synchronize()
        barrier(world)
    ms = max_over_ranks(e0.elapsed_time(e1) / steps, world)
    if rank != 0:
        return
    hbm, peak_src = peaks()
    b_alg = bytes_alg(cfg, conv)  # whole problem; per GPU it is / world
    lay = slab.layout(x, rank=rank, world=world)
    line = {
        "metric": METRIC, "value": batch / (ms / 1e3), "unit": "samples/s", "n_gpus": world, "steps": steps,
        "warmup": warm, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic (seeded N(0,1) input, seeded complex weights; no dataset)",
        "config": {"workload": desc, "global_batch": batch, "grid": list(grid), "channels": [ci, co],
                   "n_modes": list(modes), "parallelism": f"slab{world}", "x_planes_per_gpu": nx,
                   "exchange_bytes_per_gpu": int(sum(lay.send1_split()) + sum(lay.send2_split()))},
        "block_roofline": {"bound": "hbm", "achieved": b_alg / world / (ms / 1e3) / 1e9, "peak": hbm,
                           "unit": "GB/s", "frac": b_alg / world / (ms / 1e3) / 1e9 / hbm,
                           "definition": "(|x| + |y| + |W| + |bias|) / n_gpus per forward over the step time",
                           "peak_source": peak_src},
        "clocks": clocks.summary(),
    }
    print(json.dumps(line), flush=True)


def cpu_baseline(cfg, seconds=12.0):
    """Oracle (reference torch CPU path) on the host cores, bounded sample of the workload."""
    import oracle
    desc, batch, ci, co, grid, modes, fact = cfg
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    sample_b = max(1, min(batch, 4 if math.prod(grid) <= 512 * 512 else 1))
    conv, x = make_inputs((desc, sample_b, ci, co, grid, modes, fact), "cpu", seed=1)
    if fact:
        w = {"core": conv.weight.core.detach(), "factors": [f.detach() for f in conv.weight.factors]}
        kind = "tucker"
    else:
        w, kind = conv.weight.tensor.detach(), "dense"
    run = lambda: oracle.spectral_conv(x, w, conv.bias.detach(), modes, weight_kind=kind)
    with torch.no_grad():
        run()  # warm-up
        t0 = time.perf_counter()
        n = 0
        while True:
            run()
            n += 1
            if time.perf_counter() - t0 >= seconds or n >= 50:
                break
        dt = (time.perf_counter() - t0) / n
    return {"value": sample_b / dt, "unit": "samples/s", "cores": threads, "kind": "port",
            "sample": f"{sample_b} of {batch} samples per forward, {n} forwards, torch {torch.__version__} CPU"}


def run_reference_layer(args, cfg, threads):
    """Reference arm of the single-layer workload: the oracle's SpectralConv forward on a sub-batch."""
    steps, warm = args.steps, args.warmup
    import oracle
    desc, batch, ci, co, grid, modes, fact = cfg
    sample_b = max(1, min(batch, 4 if math.prod(grid) <= 512 * 512 else 1))
    conv, x = make_inputs((desc, sample_b, ci, co, grid, modes, fact), "cpu", seed=1)
    if fact:
        w = {"core": conv.weight.core.detach(), "factors": [f.detach() for f in conv.weight.factors]}
        kind = "tucker"
    else:
        w, kind = conv.weight.tensor.detach(), "dense"
    with torch.no_grad():
        for _ in range(warm):
            oracle.spectral_conv(x, w, conv.bias.detach(), modes, weight_kind=kind)
        t0 = time.perf_counter()
        for _ in range(steps):
            oracle.spectral_conv(x, w, conv.bias.detach(), modes, weight_kind=kind)
        dt = (time.perf_counter() - t0) / steps
    value = sample_b / dt
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "samples/s", "n_gpus": args.gpus,
            "steps": steps, "warmup": warm, "ms_per_step": dt * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": desc, "global_batch": batch, "sample_batch": sample_b, "grid": list(grid),
                       "channels": [ci, co], "n_modes": list(modes), "parallelism": "cpu"},
            "cpu_baseline": {"value": value, "unit": "samples/s", "cores": threads, "kind": "port",
                             "sample": f"{sample_b} of {batch} samples per step (oracle = reference torch CPU path)"},
            "e2e": {"value": value, "unit": "samples/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def _oracle_stages(model, cfg, x):
    """The oracle's FNO forward (oracle.fno_forward: fno.py:342-408) cut into four stages of similar cost:
    [grid embedding + lifting + block 0], [block 1], [block 2], [block 3 + projection].  Returns a list of
    callables h -> h."""
    import oracle
    params, ocfg = oracle_params(model)
    n = len(params["blocks"])

    def stage(first, last):
        def run(h):
            if first == 0:
                h = oracle.grid_embedding(h)
                h = oracle.channel_mlp(h, params["lifting"])
            for i in range(first, last):
                h = oracle.fno_block(h, params["blocks"][i], i, n, ocfg)
            if last == n:
                h = oracle.channel_mlp(h, params["projection"])
            return h
        return run

    bounds = [(0, 1), (1, 2), (2, 3), (3, n)] if n == 4 else [(0, n)]
    return [stage(a, b) for a, b in bounds]


def cpu_baseline_model(cfg_name, model, seconds=None):
    """The oracle (the reference's FNO forward restated on the CPU with torch) on every host core, on one
    sample of the configuration (1 sample is the bounded sample; its time is per sample)."""
    desc, cls, modes, hidden, cin, cout, grid, batch, kw, field = MODELS[cfg_name]
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    x = grf(1, cin, grid, field, seed=1, device="cpu")
    stages = _oracle_stages(model, None, x)
    with torch.no_grad():
        t0 = time.perf_counter()
        h = x
        for st in stages:
            h = st(h)
        dt = time.perf_counter() - t0
    return {"value": 1.0 / dt, "unit": "samples/s", "cores": threads, "kind": "port",
            "sample": f"1 of {batch} samples, one full forward ({dt:.1f} s), torch {torch.__version__} CPU, "
                      f"{threads} threads"}


def run_reference(args, world, rank):
    """The reference arm: the reference's own CPU path for the forward (the oracle restates it; the
    reference package cannot be imported here -- tensorly / tensorly-torch / opt-einsum are absent) on all
    host threads, on rank 0 only.  FNO: each step runs one of the forward's four stages on one sample
    (lifting + block 0, block 1, block 2, block 3 + projection, in turn) so a step stays a few seconds;
    samples/s = 1 / (sum over the stages of their mean step time).  Layer: each step is one SpectralConv
    forward on a bounded sub-batch."""
    if rank != 0:
        return
    steps, warm = args.steps, args.warmup
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    if args.model == "layer":
        run_reference_layer(args, CONFIGS[args.config] if args.batch is None else
                            (CONFIGS[args.config][0], args.batch) + tuple(CONFIGS[args.config][2:]), threads)
        return
    desc, cls, modes, hidden, cin, cout, grid, batch, kw, field = MODELS[args.config]
    model = build_model(args.config, "cpu", args.precision)
    x = grf(1, cin, grid, field, seed=1, device="cpu")
    stages = _oracle_stages(model, None, x)
    ns = len(stages)
    inputs = [x] + [None] * (ns - 1)
    times = [[] for _ in range(ns)]
    budget_s = args.reference_seconds
    t_start = time.perf_counter()
    done = 0
    with torch.no_grad():
        # warm-up steps run the stages in order, which also produces every stage's input
        for k in range(max(warm, ns)):
            j = k % ns
            h = stages[j](inputs[j])
            if j + 1 < ns and inputs[j + 1] is None:
                inputs[j + 1] = h
        for k in range(steps):
            j = k % ns
            t0 = time.perf_counter()
            stages[j](inputs[j])
            times[j].append(time.perf_counter() - t0)
            done += 1
            if time.perf_counter() - t_start > budget_s and all(times):
                break
    per_sample = sum(statistics.mean(t) for t in times if t) * ns / sum(1 for t in times if t)
    value = 1.0 / per_sample
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "samples/s", "n_gpus": args.gpus,
            "steps": done, "warmup": max(warm, ns), "ms_per_step": per_sample / ns * 1e3, "higher_is_better": True,
            "scaling": "strong" if (args.gpus > 1 and len(grid) == 3) else "weak", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic (the same seeded random field and seeded random-init weights)",
            "config": {"workload": f"{desc}_forward", "model": cls, "global_batch": batch, "sample_batch": 1,
                       "grid": list(grid), "hidden_channels": hidden, "n_modes": list(modes), "parallelism": "cpu",
                       "stage_ms": [statistics.mean(t) * 1e3 if t else None for t in times],
                       "steps_requested": steps, **{k: v for k, v in kw.items()}},
            "cpu_baseline": {"value": value, "unit": "samples/s", "cores": threads, "kind": "port",
                             "sample": f"1 of {batch} samples; each step one quarter of the forward (lifting + "
                                       f"block 0, block 1, block 2, block 3 + projection in turn); {done} timed "
                                       f"steps within a {budget_s:.0f} s budget (oracle = reference torch CPU "
                                       f"path, torch {torch.__version__})"},
            "e2e": {"value": value, "unit": "samples/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def kernel_names(plan, cfg):
    """Names of the kernels one forward launches, in launch order (fused engine layouts)."""
    fact = cfg[6]
    mix = ["contraction"] if not fact else ["contraction_in_factor", "contraction_core", "contraction_out_factor"]
    nd = len(cfg[4])
    if not plan.is_fast:
        return [f"kernel_{i}" for i in range(plan.launches_per_forward)]
    if nd == 3:
        return ["plane_fwd", "axis_fwd"] + mix + ["axis_inv", "plane_inv"]
    if nd == 1:
        return ["row_fwd"] + mix + ["row_inv"]
    return ["plane_fwd"] + mix + ["plane_inv"]


def kernel_names_for(conv, cfg):
    """kernel_names for the plan a SpectralConv uses on the layer configuration ``cfg``."""
    from neuraloperator_b200 import ops
    desc, batch, ci, co, grid, modes, fact = cfg
    geo = conv.geometry(list(grid))
    kind, _, ranks = conv.kernel_operands(geo)
    plan = ops.get_plan(ops.make_desc(geo, batch, ci, co, weight_kind=kind, ranks=ranks,
                                      precision=conv.contraction_precision, engine=conv.engine),
                        torch.cuda.current_device())
    return kernel_names(plan, cfg)


def kernel_bytes(name, cfg, conv):
    """Compulsory HBM bytes of one kernel launch: its inputs and outputs, each touched once."""
    _, batch, ci, co, grid, modes, _ = cfg
    p = math.prod(grid)
    geo = conv.geometry(list(grid))
    mt = geo.n_modes_total
    xs, ys = batch * ci * mt * 8, batch * co * mt * 8
    w = sum(t.numel() * t.element_size() for t in conv.weight.parameters())
    plane_modes = mt // geo.kept[0] if len(grid) == 3 else mt
    table = {
        "plane_fwd": batch * ci * p * 4 + (batch * ci * grid[0] * plane_modes * 8 if len(grid) == 3 else xs),
        "row_fwd": batch * ci * p * 4 + xs,
        "plane_inv": (batch * co * grid[0] * plane_modes * 8 if len(grid) == 3 else ys) + batch * co * p * 4,
        "row_inv": ys + batch * co * p * 4,
        "axis_fwd": batch * ci * grid[0] * plane_modes * 8 + xs,
        "axis_inv": ys + batch * co * grid[0] * plane_modes * 8,
        "contraction": xs + w + ys,
    }
    return table.get(name)


def run_ours(args, cfg, world, rank, local):
    import neuraloperator_b200 as nb  # noqa: F401
    from neuraloperator_b200 import ops

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    desc, batch, ci, co, grid, modes, fact = cfg
    conv, x = make_inputs(cfg, dev, seed=0)
    conv.engine = args.engine
    conv.contraction_precision = args.precision
    stream = torch.cuda.current_stream(dev)
    steps, warm = args.steps, args.warmup

    with torch.no_grad():
        for _ in range(warm):
            y = conv(x)
        torch.cuda.synchronize()
        geo = conv.geometry(list(grid))
        kind, _, ranks = conv.kernel_operands(geo)
        desc_c = ops.make_desc(geo, batch, ci, co, weight_kind=kind, ranks=ranks, precision=args.precision,
                               engine=args.engine)
        plan = ops.get_plan(desc_c, local)

        # ---- per-kernel device times (CUDA events recorded by the library on the launching stream) ----
        from neuraloperator_b200 import _lib
        nk = plan.launches_per_forward
        marks = [_lib.LaunchEvents(nk) for _ in range(steps)]
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier(world)
        torch.cuda.synchronize()
        e0.record(stream)
        for k in range(steps):
            with marks[k]:
                y = conv(x)
        e1.record(stream)
        torch.cuda.synchronize()
        ms_eager = max_over_ranks(e0.elapsed_time(e1) / steps, world)
        per_kernel = [statistics.mean(m.durations_ms()[i] for m in marks) for i in range(nk)]

        # ---- timed region: K forwards replayed from one captured CUDA graph (the same kernels with
        # the host launch overhead removed); eager launches when capture is off or fails ----
        graph, launch = None, "eager"
        if not args.no_graph:
            graph, launch = capture_graph(lambda: conv(x), stream)
        barrier(world)
        torch.cuda.synchronize()
        with ClockSampler(local) as clocks:
            e0.record(stream)
            for _ in range(steps):
                if graph is not None:
                    graph.replay()
                else:
                    y = conv(x)
            e1.record(stream)
            torch.cuda.synchronize()
        barrier(world)
        ms = max_over_ranks(e0.elapsed_time(e1) / steps, world)
        value = world * batch / (ms / 1e3)
        del graph

        e2e_how = None
        if args.no_e2e:
            ms_e2e = float("nan")
        else:
            ms_e2e = None
    if ms_e2e is None:
        # ---- end to end through the public API: pinned host in, pinned host out.  forward_host
        # (nop_spectral_forward_host) cuts the batch into chunks whose H2D copy, kernels and D2H copy
        # overlap across streams; every byte of x and y still crosses PCIe inside the timed region.
        x_host = x.cpu().pin_memory()
        y_host = torch.empty(y.shape, dtype=y.dtype).pin_memory()
        chunk = ops.default_chunk(batch)
        e2e_steps = max(1, min(steps, 10))
        with torch.no_grad():
            conv.forward_host(x_host, out=y_host, chunk=chunk, n_streams=E2E_STREAMS)  # plan + packing
            barrier(world)
            torch.cuda.synchronize()
            f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            f0.record(stream)
            for _ in range(e2e_steps):
                conv.forward_host(x_host, out=y_host, chunk=chunk, n_streams=E2E_STREAMS, synchronize=False)
            f1.record(stream)
        torch.cuda.synchronize()
        barrier(world)
        ms_e2e = max_over_ranks(f0.elapsed_time(f1) / e2e_steps, world)
        e2e_how = (f"SpectralConv.forward_host (nop_spectral_forward_host): {batch // chunk} chunks of {chunk} "
                   f"samples over {E2E_STREAMS} streams, pinned host buffers")

    if rank != 0:
        return
    hbm, peak_src = peaks()
    b_alg = bytes_alg(cfg, conv)
    block_gbs = b_alg / (ms / 1e3) / 1e9
    clk = clocks.summary()
    names = kernel_names(plan, cfg)
    kernels = []
    for name, kms in zip(names, per_kernel):
        kb = kernel_bytes(name, cfg, conv)
        kernels.append({"name": name, "ms": kms, "bytes_alg": kb,
                        "gbs": kb / (kms / 1e3) / 1e9 if kb else None,
                        "frac": kb / (kms / 1e3) / 1e9 / hbm if kb else None})
    dom = max(kernels, key=lambda k: k["ms"])
    line = {
        "metric": METRIC, "value": value, "unit": "samples/s", "n_gpus": world, "steps": steps, "warmup": warm,
        "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32" if args.precision == "fp32" else "f32 (bf16 contraction)",
        "data": "synthetic (seeded N(0,1) input, seeded complex weights; no dataset)",
        "config": {"workload": desc, "global_batch": batch * world, "per_gpu_batch": batch, "grid": list(grid),
                   "channels": [ci, co], "n_modes": list(modes), "factorization": fact or "dense",
                   "parallelism": f"dp{world}" if world > 1 else "single", "engine": "fast" if plan.is_fast else
                   "generic", "l2": f"inputs {x.numel() * 4 / 1e9:.2f} GB > 126 MB L2 (no flush needed)",
                   "launch": launch, "ms_per_step_eager": ms_eager},
        "roofline": {"bound": "hbm", "achieved": dom["gbs"], "peak": hbm, "unit": "GB/s", "frac": dom["frac"],
                     "traffic": TRAFFIC.get((args.config, dom["name"])), "kernel": dom["name"],
                     "bytes_alg_per_launch": dom["bytes_alg"], "ms_per_launch": dom["ms"],
                     "peak_source": peak_src + " (copy bandwidth, burst)"},
        "block_roofline": {"bound": "hbm", "achieved": block_gbs, "peak": hbm, "unit": "GB/s",
                           "frac": block_gbs / hbm, "bytes_alg_per_step": b_alg,
                           "definition": "|x| + |y| + |W| + |bias| per forward over the step time"},
        "kernels": kernels,
        "e2e": ({"value": world * batch / (ms_e2e / 1e3), "unit": "samples/s",
                 "h2d_bytes_per_step": x.numel() * x.element_size(),
                 "d2h_bytes_per_step": y.numel() * y.element_size(), "path": e2e_how} if not args.no_e2e else None),
        "gpu_launches": plan.launches_per_forward * steps,
        "clocks": clk,
    }
    if not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(cfg, seconds=args.cpu_seconds)
    print(json.dumps(line), flush=True)


def run_train(args, cfg, world, rank, local):
    """One SpectralConv training step at the config's size: the forward (keeping the kept input spectrum)
    and the backward giving dL/dx, dL/dW and dL/dbias for a fixed dL/dy, through torch autograd and the
    library's kernels (neuralop/training/trainer.py:629-700 runs forward + loss.backward() per batch).
    Every rank runs its own batch (weak scaling).  The phases are also timed one by one (rank 0)."""
    from neuraloperator_b200 import _lib, ops
    from neuraloperator_b200.geometry import adjoint_geometry

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    desc, batch, ci, co, grid, modes, fact = cfg
    conv, x = make_inputs(cfg, dev, seed=0)
    conv.engine = args.engine
    conv.contraction_precision = args.precision
    x.requires_grad_(True)
    params = list(conv.parameters())
    gen = torch.Generator(device="cpu").manual_seed(1)
    g = torch.randn((batch, co, *grid), generator=gen).to(dev)
    stream = torch.cuda.current_stream(dev)
    steps, warm = args.steps, args.warmup

    def step():
        y = conv(x)
        return torch.autograd.grad(y, [x] + params, g)

    for _ in range(warm):
        step()
    torch.cuda.synchronize()
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        grads = step()
    e1.record(stream)
    torch.cuda.synchronize()
    ms_eager = max_over_ranks(e0.elapsed_time(e1) / steps, world)
    del grads
    # timed region: the whole step (forward, autograd backward, every kernel of both) replayed from one
    # CUDA graph, which removes the Python / autograd host time between launches; eager if capture fails
    graph, launch = None, "eager"
    if not args.no_graph:
        try:
            graph = torch.cuda.CUDAGraph()
            side = torch.cuda.Stream()
            side.wait_stream(stream)
            with torch.cuda.stream(side):
                step()
                with torch.cuda.graph(graph, stream=side):
                    grads = step()
            stream.wait_stream(side)
            torch.cuda.synchronize()
            launch = "cuda_graph"
        except Exception as exc:  # noqa: BLE001
            print(f"graph capture failed, timing eager launches: {exc}", file=sys.stderr)
            graph = None
            torch.cuda.synchronize()
    barrier(world)
    with ClockSampler(local) as clocks:
        e0.record(stream)
        for _ in range(steps):
            if graph is not None:
                graph.replay()
            else:
                step()
        e1.record(stream)
        torch.cuda.synchronize()
    barrier(world)
    ms = max_over_ranks(e0.elapsed_time(e1) / steps, world)
    del graph
    if rank != 0:
        return

    def timed(fn, n=max(3, min(steps, 20))):
        """Device time of one phase, replayed from a CUDA graph like the step (eager launches would add
        the Python host time between them); eager if capture fails."""
        out = fn()
        torch.cuda.synchronize()
        g_phase = None
        if not args.no_graph:
            try:
                g_phase = torch.cuda.CUDAGraph()
                side = torch.cuda.Stream()
                side.wait_stream(stream)
                with torch.cuda.stream(side):
                    with torch.cuda.graph(g_phase, stream=side):
                        out = fn()
                stream.wait_stream(side)
                torch.cuda.synchronize()
            except Exception:  # noqa: BLE001
                g_phase = None
                torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(n):
            if g_phase is not None:
                g_phase.replay()
            else:
                out = fn()
        b.record(stream)
        torch.cuda.synchronize()
        return a.elapsed_time(b) / n, out

    geo = conv.geometry(list(grid))
    kind, ws, ranks = conv.kernel_operands(geo)
    ws = [w.detach() for w in ws]
    xd = x.detach()
    ms_fwd, (_, spec) = timed(lambda: ops.spectral_forward(xd, geo, ws, out_channels=co, weight_kind=kind, ranks=ranks,
                                                            precision=args.precision, engine=args.engine,
                                                            keep_spectrum=True))
    adj = adjoint_geometry(geo)
    packed_adj = None
    if kind == "dense":  # the backward packs the adjoint straight from W (conjugate transpose in the pack)
        ms_ops, packed_adj = timed(lambda: ops.pack_adjoint_dense(adj, batch, ws[0], precision=args.precision,
                                                                   engine=args.engine))
        aw, ar = [], ()
    else:
        ms_ops, (aw, ar) = timed(lambda: ops.adjoint_operands(kind, ws, ranks, False))
    ms_adj, (_, gspec) = timed(lambda: ops.spectral_forward(g, adj, aw, out_channels=ci, weight_kind=kind, ranks=ar,
                                                             precision=args.precision, engine=args.engine,
                                                             keep_spectrum=True, packed=packed_adj))
    wshape = (ci, co) + tuple(geo.kept)
    ms_wg, (gw, _) = timed(lambda: ops.weight_grad(spec, gspec, wshape, co))
    marks = _lib.LaunchEvents(3)  # the weight-gradient kernel alone, one eager call
    with marks:
        ops.weight_grad(spec, gspec, wshape, co)
    torch.cuda.synchronize()
    wg_kernel_ms = marks.durations_ms()[0]
    ms_fac = 0.0
    if kind == "tucker":
        from neuraloperator_b200.spectral_convolution import _tucker_grads
        ms_fac, _ = timed(lambda: _tucker_grads(ws[0], ws[1:], gw))

    hbm, peak_src = peaks()
    p = math.prod(grid)
    w_bytes = sum(t.numel() * t.element_size() for t in conv.weight.parameters())
    mt = math.prod(geo.kept)
    # algorithmic bytes of a training step: x, y (forward), dL/dy, dL/dx (backward), W twice, dL/dW, bias
    b_alg = 2 * batch * ci * p * 4 + 2 * batch * co * p * 4 + 2 * w_bytes + w_bytes + 2 * co * 4
    wg_bytes = (batch * ci * mt + batch * co * mt + ci * co * mt) * 8
    wg_flop = 8 * batch * ci * co * mt
    plan_f = ops.get_plan(ops.make_desc(geo, batch, ci, co, weight_kind=kind, ranks=ranks, precision=args.precision,
                                        engine=args.engine), local)
    plan_a = ops.get_plan(ops.make_desc(adj, batch, co, ci, weight_kind=kind, ranks=ar, precision=args.precision,
                                        engine=args.engine), local)
    pack = (1 if kind == "dense" else 3 + len(geo.kept)) if plan_a.packed_bytes > 0 else 0
    launches = plan_f.launches_per_forward + pack + plan_a.launches_per_forward + 2
    if kind == "tucker":  # nop_tucker_grads: one mode product per projected mode, conj(core), gram + sum per factor
        nm = len(ws) - 1
        nl, nr = nm // 2, nm - nm // 2
        launches += (nr + 2 * nl + nl * (nl - 1) + nr * (nr - 1)) + 1 + 2 * nm
    gbs = b_alg / (ms / 1e3) / 1e9
    line = {
        "metric": "SpectralConv training step (forward + backward) samples/s", "value": world * batch / (ms / 1e3),
        "unit": "samples/s", "n_gpus": world, "steps": steps, "warmup": warm, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32" if args.precision == "fp32" else "f32 (bf16 contraction)",
        "data": "synthetic (seeded N(0,1) input and dL/dy, seeded complex weights; no dataset)",
        "config": {"workload": desc + "_train", "global_batch": batch * world, "per_gpu_batch": batch,
                   "grid": list(grid), "channels": [ci, co], "n_modes": list(modes), "factorization": fact or "dense",
                   "parallelism": f"dp{world}" if world > 1 else "single",
                   "engine": "fast" if plan_f.is_fast else "generic", "launch": launch,
                   "ms_per_step_eager": ms_eager,
                   "l2": f"inputs {x.numel() * 4 / 1e9:.2f} GB > 126 MB L2 (no flush needed)"},
        "roofline": {"bound": "hbm", "achieved": gbs, "peak": hbm, "unit": "GB/s", "frac": gbs / hbm,
                     "bytes_alg_per_step": b_alg, "peak_source": peak_src + " (copy bandwidth, burst)",
                     "definition": "2|x| + 2|y| (x, y, dL/dy, dL/dx) + 2|W| + |dL/dW| + 2|bias| over the step time"},
        "phases_ms": {"forward_keep_spectrum": ms_fwd, "adjoint_weights": ms_ops, "adjoint_forward": ms_adj,
                      "weight_grad": ms_wg, "tucker_factor_grads": ms_fac},
        "weight_grad_kernel": {"ms": wg_kernel_ms, "bytes_alg": wg_bytes,
                               "gbs": wg_bytes / (wg_kernel_ms / 1e3) / 1e9, "tflops": wg_flop / (wg_kernel_ms / 1e3) / 1e12,
                               "definition": "|Xh| + |Gh| + |dL/dW| bytes; 8 B Ci Co Mt flops (fp32 FMA)"},
        "gpu_launches": launches * steps,
        "clocks": clocks.summary(),
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--model", choices=["fno", "layer"], default="fno",
                    help="fno: the whole FNO / TFNO forward (the headline); layer: one SpectralConv")
    ap.add_argument("--config", choices=sorted(CONFIGS), default=None,
                    help="default c5 (FNO 3D, the largest single-GPU configuration) for --model fno, c2 for layer")
    ap.add_argument("--engine", choices=["auto", "fast", "generic"], default="auto")
    ap.add_argument("--batch", type=int, default=None, help="per-GPU batch (default: the config's)")
    ap.add_argument("--grid", type=int, default=None,
                    help="--model fno: points per axis instead of the config's (small profiling cases only)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--reference-seconds", type=float, default=240.0,
                    help="time budget of the reference arm's timed steps (the FNO stages take seconds each)")
    ap.add_argument("--no-slab-check", dest="slab_check", action="store_false",
                    help="skip rank 0's comparison of its slab with a single-GPU forward")
    ap.add_argument("--no-graph", action="store_true", help="time eager launches instead of graph replay")
    ap.add_argument("--precision", choices=["fp32", "bf16"], default="fp32", help="contraction precision")
    ap.add_argument("--parallel", choices=["batch", "slab"], default="batch",
                    help="--model layer only: batch (each rank its own batch, weak) or slab (3D x split, strong)")
    ap.add_argument("--pass", dest="pass_", choices=["forward", "train"], default="forward",
                    help="--model layer only: forward, or train (forward + backward of one layer)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.config is None:
        args.config = "c5" if args.model == "fno" else "c2"
    if args.model == "fno" and args.config == "c2":
        raise SystemExit("c2 is the single-SpectralConv microbench: use --model layer")
    if args.impl == "reference":
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        run_reference(args, world, rank)
        return
    cfg = CONFIGS[args.config]
    if args.batch is not None:
        cfg = (cfg[0], args.batch) + tuple(cfg[2:])
    world, rank, local = dist_setup()
    try:
        if args.model == "fno" and args.pass_ == "train":
            run_model_train(args, world, rank, local)
        elif args.model == "fno":
            run_model(args, world, rank, local)
        elif args.pass_ == "train":
            run_train(args, cfg, world, rank, local)
        elif args.parallel == "slab":
            run_slab(args, cfg, world, rank, local)
        else:
            run_ours(args, cfg, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
