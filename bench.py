"""Benchmarks of the packed-ensemble hot path on B200.

Default workload (`--workload train`): full TabPack training of the full-training
configuration -- a global pack of 512 members (depth U{1..4}, width U{128..1024}, dropout
U[0, 0.5]) on 1 000 000 synthetic rows with 100 numerical and 10 categorical features,
batch 1024, BCE, Muon + AdamW, bf16 autocast -- with the members sharded over the GPUs
(contiguous ranges balanced by FLOPs per step; strong scaling).  The timed region is an
epoch scaled to K steps: K training steps over the first K x 1024 rows, then the epoch end
over the first K / 977 of the 100 000 validation rows (every member's predictions
all-gathered over NCCL, a greedy ensemble built from them).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference] [--workload ...]

Prints one JSON line (rank 0).  `value` is whole-job member-samples/s with the data resident
in HBM; `e2e` repeats the region through the same public calls with the step inputs copied
from pinned host memory and the losses and gathered predictions read back; `roofline` covers
the kernel family with the largest share of the step (per-launch CUDA-event times from the
library's profiler, `tp_profile_start` / `tp_profile_stop`); `config.checksum` hashes the
trained pack's gathered validation predictions (equal at every N when sharding does not change
the arithmetic); `cpu_baseline` and `--impl reference` time the reference's training step
restated with the reference's own torch ops on the host cores, on a member sample.

Other workloads (`--workload`): `layer` (one packed MLP block forward + backward: 256
members per GPU over a shared 4096 x 512 bf16 batch), `optimizer`, `metrics`, `inference`,
`onehot`; each prints its own JSON line.
"""

from __future__ import annotations

import argparse
import ctypes
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

MEMBERS = 256
ROWS = 4096
D_IN = 512
MAX_OUT = 1024
WORKLOAD = ('packed MLP block forward+backward: 256 members/GPU sharing a 4096x512 bf16 batch, '
            'out widths U{64..1024 step 16}, bias + ReLU + Philox dropout p~U[0,0.5], fp32 accumulation; '
            'output buffer reused across steps (its zero padding written once)')


def member_widths(base: int, n: int) -> np.ndarray:
    """Per-member output widths, seeded by global member id (shard-invariant)."""
    out = np.empty(n, np.int32)
    for i in range(n):
        out[i] = np.random.default_rng(1_000_003 * (base + i) + 7).integers(4, 65) * 16
    return out


def member_dropout(base: int, n: int) -> np.ndarray:
    return np.array([np.random.default_rng(7_000_001 * (base + i) + 3).uniform(0, 0.5) for i in range(n)], np.float32)


def peak_key(clk: dict) -> str:
    """The bf16 peak that applies to a timed region: the sustained figure when the SM clock ran
    below 90 % of its maximum there (the power cap held it down), the burst figure otherwise."""
    if clk.get('sm_mhz') and clk.get('sm_max_mhz') and clk['sm_mhz'] < 0.9 * clk['sm_max_mhz']:
        return 'bf16_tflops_sustained'
    return 'bf16_tflops'


def load_peaks() -> tuple[dict, str]:
    path = os.path.join(ROOT, 'MEASURED_PEAKS.json')
    if os.path.exists(path):
        with open(path) as f:
            return json.load(f), 'measured'
    return {'hbm_gbs': 6650.0, 'bf16_tflops': 1590.0, 'bf16_tflops_sustained': 1400.0}, 'fallback'


def dist_init(dev, seconds: int = 300) -> int:
    """Joins the NCCL process group once (torchrun's env); returns the world size."""
    import datetime

    import torch.distributed as dist

    world = int(os.environ.get('WORLD_SIZE', '1'))
    if world > 1 and not dist.is_initialized():
        dist.init_process_group('nccl', device_id=dev, timeout=datetime.timedelta(seconds=seconds))
    return world


def dist_done(emit: bool) -> None:
    """Leaves the process group after a workload that printed its own line."""
    import torch.distributed as dist

    if emit and dist.is_initialized():
        dist.destroy_process_group()


# ----------------------------------------------------------------------------- CPU legs


def cpu_sample(members: int, budget_s: float, steps: int | None = None):
    """The reference's block forward+backward on the host (`oracle.torch_step.block_step`: padded
    baddbmm, bernoulli_ dropout, autograd; all host threads) on `members` members of the layer
    workload; returns (member-samples/s, threads, sample)."""
    import torch

    from oracle.torch_step import block_step

    torch.set_num_threads(os.cpu_count() or 1)
    g = torch.Generator().manual_seed(0)
    out_f = torch.from_numpy(member_widths(0, members))
    max_out = int(out_f.max())
    x = torch.randn(ROWS, D_IN, generator=g)
    w = (torch.rand(members, max_out, D_IN, generator=g) * 2 - 1) / D_IN ** 0.5
    b = (torch.rand(members, max_out, generator=g) * 2 - 1) / D_IN ** 0.5
    p = torch.from_numpy(member_dropout(0, members))
    dy = torch.randn(members, ROWS, max_out, generator=g)
    block_step(x, w, b, out_f, p, dy)  # warm-up
    n, t0 = 0, time.perf_counter()
    while True:
        block_step(x, w, b, out_f, p, dy)
        n += 1
        el = time.perf_counter() - t0
        if (steps is not None and n >= steps) or (steps is None and el >= budget_s):
            break
    sample = (f'{members} members x {ROWS} rows x {D_IN} in (out widths {int(out_f.sum())} total), {n} fwd+bwd steps '
              '(torch CPU restatement of the reference block: padded baddbmm, bernoulli_ dropout, autograd, fp32)')
    return members * ROWS * n / el, torch.get_num_threads(), sample


def run_reference(args) -> None:
    """The reference arm of the layer workload (rank 0 only)."""
    if int(os.environ.get('RANK', '0')) != 0:
        return
    members = 4
    for _ in range(max(args.warmup, 0)):
        cpu_sample(members, 0, steps=1)
    vals = []
    threads, sample = 1, ''
    for _ in range(args.steps):
        v, threads, sample = cpu_sample(members, 0, steps=1)
        vals.append(v)
    value = statistics.median(vals)
    line = {
        'metric': 'member-samples/sec train (packed MLP block fwd+bwd)', 'value': value,
        'unit': 'member-samples/s', 'n_gpus': args.gpus, 'steps': args.steps, 'warmup': args.warmup,
        'ms_per_step': members * ROWS / value * 1e3, 'higher_is_better': True, 'scaling': 'weak',
        'vs_baseline': None, 'dtype': 'f32', 'data': 'synthetic', 'impl': 'reference',
        'config': {'workload': WORKLOAD, 'sample_members': members},
        'cpu_baseline': {'value': value, 'unit': 'member-samples/s', 'cores': threads, 'kind': 'port',
                         'sample': sample + ', one per timed step'},
        'e2e': {'value': value, 'unit': 'member-samples/s', 'h2d_bytes_per_step': 0, 'd2h_bytes_per_step': 0},
    }
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------- clocks


class ClockSampler:
    FIELDS = ('clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,'
              'clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,'
              'clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap')

    def __init__(self, device: int) -> None:
        self.device = device
        self.lines: list[str] = []
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ['nvidia-smi', '-i', str(self.device), f'--query-gpu={self.FIELDS}', '--format=csv,noheader,nounits',
                 '-lms', '100'], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        sm, mx, reasons = [], 0.0, set()
        names = ['hw_slowdown', 'hw_thermal_slowdown', 'sw_thermal_slowdown', 'sw_power_cap']
        for ln in self.lines:
            parts = [x.strip() for x in ln.split(',')]
            if len(parts) < 8:
                continue
            try:
                sm.append(float(parts[0]))
                mx = max(mx, float(parts[1]))
            except ValueError:
                continue
            for n, v in zip(names, parts[4:8]):
                if v.lower() == 'active':
                    reasons.add(n)
        return {'sm_mhz': statistics.median(sm) if sm else None, 'sm_max_mhz': mx or None,
                'reasons': sorted(reasons), 'samples': len(sm)}


# ----------------------------------------------------------------------------- GPU leg


def run_b200(args, emit: bool = True) -> dict | None:
    """The layer workload (one packed MLP block forward + backward); prints its JSON line (rank
    0) or, with emit=False, returns it (rank 0; None elsewhere)."""
    import torch
    import torch.distributed as dist

    from tabpack_b200 import _lib

    rank = int(os.environ.get('RANK', '0'))
    local = int(os.environ.get('LOCAL_RANK', '0'))
    torch.cuda.set_device(local)
    dev = torch.device('cuda', local)
    world = dist_init(dev)
    lib = _lib.load()

    base = rank * MEMBERS
    out_f = member_widths(base, MEMBERS)
    p = member_dropout(base, MEMBERS)
    g = torch.Generator(device=dev).manual_seed(1234 + rank)
    x = torch.randn(ROWS, D_IN, device=dev, generator=g).bfloat16()
    w = ((torch.rand(MEMBERS, MAX_OUT, D_IN, device=dev, generator=g) * 2 - 1) / D_IN ** 0.5).bfloat16()
    bias = (torch.rand(MEMBERS, MAX_OUT, device=dev, generator=g) * 2 - 1) / D_IN ** 0.5
    dy = torch.randn(MEMBERS, ROWS, MAX_OUT, device=dev, generator=g).bfloat16()
    of = torch.from_numpy(out_f).to(dev)
    pd = torch.from_numpy(p).to(dev)
    # y is reused by every step: its padding is written once (zeros here), so the forwards
    # write only the members' columns (y_pad_zero)
    y = torch.zeros(MEMBERS, ROWS, MAX_OUT, device=dev, dtype=torch.bfloat16)
    gbuf = torch.empty_like(y)
    dx = torch.empty(MEMBERS, ROWS, D_IN, device=dev, dtype=torch.bfloat16)
    dw = torch.empty(MEMBERS, MAX_OUT, D_IN, device=dev, dtype=torch.float32)
    db = torch.empty(MEMBERS, MAX_OUT, device=dev, dtype=torch.float32)

    fa = _lib.LinearArgs()
    fa.P, fa.B, fa.max_in, fa.max_out = MEMBERS, ROWS, D_IN, MAX_OUT
    fa.dtype, fa.x_shared = _lib.TP_DTYPE_BF16, 1
    fa.in_features, fa.out_features, fa.n_blocks = None, of.data_ptr(), None
    fa.relu, fa.dropout_p, fa.seed, fa.member_base = 1, pd.data_ptr(), 0x5EED, base
    fa.x, fa.w, fa.bias, fa.y = x.data_ptr(), w.data_ptr(), bias.data_ptr(), y.data_ptr()
    fa.y_pad_zero = 1

    def grad_args(**kw):
        ga = _lib.LinearGradArgs()
        ga.fwd = fa
        ga.dy, ga.y, ga.g = dy.data_ptr(), y.data_ptr(), gbuf.data_ptr()
        ga.dw_rows, ga.dw_cols, ga.db_cols = MAX_OUT, D_IN, MAX_OUT
        for k, v in kw.items():
            setattr(ga, k, v)
        return ga

    ga_act = grad_args(dbias=db.data_ptr())
    ga_dx = grad_args(dx=dx.data_ptr(), g_ready=1)
    ga_dw = grad_args(dw=dw.data_ptr(), g_ready=1)
    stream = torch.cuda.current_stream(dev)
    sp = stream.cuda_stream
    phases = ['fwd', 'act', 'dgrad', 'wgrad']

    def check(rc, what):
        if rc != 0:
            raise RuntimeError(f'{what}: {lib.tp_last_error_string().decode()}')

    def step(i, ev=None):
        fa.offset = i
        ga_act.fwd.offset = i
        if ev is not None:
            ev[0].record(stream)
        check(lib.tp_linear_forward(ctypes.byref(fa), sp), 'forward')
        if ev is not None:
            ev[1].record(stream)
        check(lib.tp_linear_backward(ctypes.byref(ga_act), sp), 'act')
        if ev is not None:
            ev[2].record(stream)
        check(lib.tp_linear_backward(ctypes.byref(ga_dx), sp), 'dgrad')
        if ev is not None:
            ev[3].record(stream)
        check(lib.tp_linear_backward(ctypes.byref(ga_dw), sp), 'wgrad')
        if ev is not None:
            ev[4].record(stream)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    events = [[torch.cuda.Event(enable_timing=True) for _ in range(5)] for _ in range(args.steps)]
    barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clocks:
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        for i in range(args.steps):
            step(args.warmup + i, events[i])
        t1.record(stream)
        torch.cuda.synchronize()
    barrier()
    elapsed_ms = t0.elapsed_time(t1)
    per_phase = {ph: statistics.mean(ev[j].elapsed_time(ev[j + 1]) for ev in events) for j, ph in enumerate(phases)}
    dev_err = lib.tp_device_error()
    if dev_err != 0:
        raise RuntimeError(f'device-side wait timed out ({dev_err})')

    # end to end: batch uploaded from pinned host memory, bias gradient read back, every step
    x_host = x.cpu().pin_memory()
    db_host = torch.empty(db.shape, dtype=db.dtype).pin_memory()
    x_dev = torch.empty_like(x)
    fa_e2e_x = x_dev.data_ptr()

    def e2e_step(i):
        x_dev.copy_(x_host, non_blocking=True)
        fa.x = fa_e2e_x
        ga_act.fwd.x = fa_e2e_x
        ga_dw.fwd.x = fa_e2e_x
        step(i)
        db_host.copy_(db, non_blocking=True)

    for i in range(args.warmup):
        e2e_step(i)
    torch.cuda.synchronize()
    barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(args.steps):
        e2e_step(i)
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    e2e_ms = e0.elapsed_time(e1)

    if world > 1:
        t = torch.tensor([elapsed_ms, e2e_ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        elapsed_ms, e2e_ms = float(t[0]), float(t[1])

    samples = world * MEMBERS * ROWS * args.steps
    value = samples / (elapsed_ms / 1e3)
    e2e_value = samples / (e2e_ms / 1e3)

    peaks, peak_kind = load_peaks()
    clk = clocks.summary()
    flops = 2.0 * ROWS * D_IN * float(out_f.sum())
    # activation-gradient kernel: reads dy and y and writes g over each member's
    # 64-column strips below out_i, bf16
    act_bytes = 3.0 * 2 * ROWS * float(sum((o + 63) // 64 * 64 for o in out_f)) + 4.0 * MEMBERS * MAX_OUT
    work = {'fwd': flops, 'dgrad': flops, 'wgrad': flops, 'act': act_bytes}
    dominant = max(per_phase, key=per_phase.get)
    if dominant == 'act':
        ach = work['act'] / (per_phase['act'] / 1e3) / 1e9
        roof = {'bound': 'hbm', 'achieved': ach, 'peak': peaks['hbm_gbs'], 'unit': 'GB/s'}
    else:
        ach = work[dominant] / (per_phase[dominant] / 1e3) / 1e12
        roof = {'bound': 'tensor', 'achieved': ach, 'peak': peaks[peak_key(clk)], 'unit': 'TFLOP/s'}
    roof['frac'] = roof['achieved'] / roof['peak']
    roof['kernel'] = dominant
    roof['traffic'] = TRAFFIC_BYTES_PER_LAUNCH.get(dominant)
    roof['peak_source'] = (f'{peak_kind} (copy)' if roof['bound'] == 'hbm' else
                           f'{peak_kind} ({peak_key(clk)}: median SM clock {clk["sm_mhz"]} of {clk["sm_max_mhz"]} MHz)')

    if rank != 0:
        dist_done(emit)
        return None

    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        v, threads, sample = cpu_sample(4, args.cpu_seconds)
        cpu = {'value': v, 'unit': 'member-samples/s', 'cores': threads, 'kind': 'port', 'sample': sample}

    tflops_step = 3 * flops * world / (elapsed_ms / args.steps / 1e3) / 1e12
    line = {
        'metric': 'member-samples/sec train (packed MLP block fwd+bwd)', 'value': value,
        'unit': 'member-samples/s', 'n_gpus': world, 'steps': args.steps, 'warmup': args.warmup,
        'ms_per_step': elapsed_ms / args.steps, 'higher_is_better': True, 'scaling': 'weak',
        'vs_baseline': None, 'dtype': 'bf16', 'data': 'synthetic',
        'config': {'workload': WORKLOAD, 'members_per_gpu': MEMBERS, 'rows': ROWS, 'd_in': D_IN,
                   'max_out': MAX_OUT, 'ragged_tflop_per_step_per_gpu': 3 * flops / 1e12,
                   'ragged_tflops_achieved': tflops_step, 'parallelism': f'member-sharded x{world}',
                   'l2': 'inputs larger than L2 (weights 256 MiB, activations 2 GiB per GPU)',
                   'per_kernel_ms': per_phase},
        'roofline': roof,
        'cpu_baseline': cpu,
        'e2e': {'value': e2e_value, 'unit': 'member-samples/s', 'h2d_bytes_per_step': x.numel() * 2,
                'd2h_bytes_per_step': db.numel() * 4},
        'gpu_launches': 4 * args.steps,
        'clocks': clk,
    }
    if emit:
        print(json.dumps(line), flush=True)
    dist_done(emit)
    return line


# DRAM bytes (read + write) per full-size launch, from the ncu capture of the layer kernels
# (32-member case scaled by 256/32).
TRAFFIC_BYTES_PER_LAUNCH: dict[str, float | None] = {
    'fwd': (25.810688e6 + 91.443712e6) * 8,
    'act': (293.625344e6 + 94.327552e6) * 8,
    'dgrad': (173.594624e6 + 100.386560e6) * 8,
    'wgrad': (180.835072e6 + 42.455808e6) * 8,
}


def run_optimizer(args, emit: bool = True) -> dict | None:
    """Grouped optimizer step: `members` x 3 weight matrices with rows and cols ~ U{64..1024
    step 16} (entries N(0, 0.02^2), gradients N(0, 1e-3^2)), one Muon group per matrix with
    5 Newton-Schulz iterations and the update scale sqrt(max(1, out/in)), plus one grouped
    AdamW launch over the matrices' bias vectors; per-member lr log-U[1e-4, 1e-2], weight
    decay log-U[1e-6, 1e-2], beta2 U[0.95, 0.999].  Also timed at this size: the Muon
    elementwise kernels (library profiler, 28 B per weight element: momentum, Nesterov blend,
    bf16 operand, normalisation, update) and a grouped AdamW step over the three weight packs
    themselves (28 B per element), each against the measured copy bandwidth.  Under torchrun
    every rank runs the whole workload on its own GPU (replicas); times are the max over
    ranks."""
    import torch
    import torch.distributed as dist

    from tabpack_b200 import ops

    rank = int(os.environ.get('RANK', '0'))
    local = int(os.environ.get('LOCAL_RANK', '0'))
    torch.cuda.set_device(local)
    dev = torch.device('cuda', local)
    world = dist_init(dev)
    P = args.members
    rng = np.random.default_rng(5)
    groups = []
    flops = 0.0
    elems = 0
    for j in range(3):
        outs = rng.integers(4, 65, P).astype(np.int32) * 16
        ins = rng.integers(4, 65, P).astype(np.int32) * 16
        mo, mi = int(outs.max()), int(ins.max())
        g = torch.Generator(device=dev).manual_seed(j)
        p = torch.zeros(P, mo, mi, device=dev)
        grad = torch.zeros_like(p)
        mask = ((torch.arange(mo, device=dev)[None, :, None] < torch.from_numpy(outs).to(dev)[:, None, None]) &
                (torch.arange(mi, device=dev)[None, None, :] < torch.from_numpy(ins).to(dev)[:, None, None]))
        p.copy_(torch.randn(P, mo, mi, device=dev, generator=g) * 0.02 * mask)
        grad.copy_(torch.randn(P, mo, mi, device=dev, generator=g) * 1e-3 * mask)
        del mask
        r = np.minimum(outs, ins).astype(np.float64)
        c = np.maximum(outs, ins).astype(np.float64)
        flops += float(np.sum(5 * (4 * r * r * c + 2 * r ** 3)))
        elems += int(np.sum(outs.astype(np.int64) * ins))
        groups.append(dict(p=p, grad=grad, m=torch.zeros_like(p), outf=torch.from_numpy(outs).to(dev),
                           inf=torch.from_numpy(ins).to(dev), ws=torch.empty(ops.muon_workspace_size(P, mo, mi),
                                                                             dtype=torch.uint8, device=dev)))
    lr = torch.from_numpy(np.exp(rng.uniform(np.log(1e-4), np.log(1e-2), P)).astype(np.float32)).to(dev)
    wd = torch.from_numpy(np.exp(rng.uniform(np.log(1e-6), np.log(1e-2), P)).astype(np.float32)).to(dev)
    beta2 = torch.from_numpy(rng.uniform(0.95, 0.999, P).astype(np.float32)).to(dev)
    mu = torch.full((P,), 0.95, device=dev)
    for gr in groups:
        gr['scale'] = torch.sqrt(torch.clamp(gr['outf'].float() / gr['inf'].float(), min=1.0))
    # AdamW state of the biases (P, max_out) of the three matrices
    biases = [dict(p=torch.randn(P, gr['p'].shape[1], device=dev) * 0.02,
                   g=torch.randn(P, gr['p'].shape[1], device=dev) * 1e-3) for gr in groups]
    for b in biases:
        b['m'], b['v'] = torch.zeros_like(b['p']), torch.zeros_like(b['p'])
    adamw_elems = sum(b['p'].numel() for b in biases)

    def step(i=0, ev=None):
        for gr in groups:
            ops.muon_step(gr['p'], gr['grad'], gr['m'], out_features=gr['outf'], in_features=gr['inf'], lr=lr,
                          momentum=mu, weight_decay=wd, update_scale=gr['scale'], nesterov=True,
                          mutate_grad=False, ns_steps=5, workspace=gr['ws'])
        if ev is not None:
            ev[0].record()
        ops.adamw_step([b['p'] for b in biases], [b['g'] for b in biases], [b['m'] for b in biases],
                       [b['v'] for b in biases], step=i + 1, lr=lr, beta1=0.9, beta2=beta2, eps=1e-8,
                       weight_decay=wd)
        if ev is not None:
            ev[1].record()

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])
        torch.cuda.synchronize()

    for i in range(args.warmup):
        step(i)
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    aev = [[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(args.steps)]
    with ClockSampler(local) as clocks:
        e0.record()
        for i in range(args.steps):
            step(args.warmup + i, aev[i])
        e1.record()
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    adamw_ms = statistics.mean(a.elapsed_time(b) for a, b in aev)
    # the Muon elementwise kernels and the Newton-Schulz GEMMs, launch by launch
    with ops.KernelTimes() as kt:
        step(args.warmup + args.steps)
    muon_el_ms = kt.ms['muon_elementwise']
    ns_ms = kt.ms['newton_schulz_gram'] + kt.ms['newton_schulz_update']
    # AdamW over the weight packs themselves (what an AdamW optimizer pack would run on them);
    # the Muon momentum buffers serve as first moments
    for b in biases:
        del b['v']
    vs = [torch.zeros_like(gr['p']) for gr in groups]
    big = dict(params=[gr['p'] for gr in groups], grads=[gr['grad'] for gr in groups],
               exp_avgs=[gr['m'] for gr in groups], exp_avg_sqs=vs)
    big_elems = sum(gr['p'].numel() for gr in groups)

    def adamw_big(i):
        ops.adamw_step(big['params'], big['grads'], big['exp_avgs'], big['exp_avg_sqs'], step=i + 1, lr=lr,
                       beta1=0.9, beta2=beta2, eps=1e-8, weight_decay=wd)

    adamw_big(0)
    torch.cuda.synchronize()
    b0, b1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    b0.record()
    for i in range(args.steps):
        adamw_big(1 + i)
    b1.record()
    torch.cuda.synchronize()
    adamw_big_ms = b0.elapsed_time(b1) / args.steps
    t = torch.tensor([ms, adamw_ms, muon_el_ms, ns_ms, adamw_big_ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, adamw_ms, muon_el_ms, ns_ms, adamw_big_ms = (float(v) for v in t)
    del groups, biases, big, vs
    if rank != 0:
        dist_done(emit)
        return None
    peaks, kind = load_peaks()
    clk = clocks.summary()
    sustained = peak_key(clk) == 'bf16_tflops_sustained'
    peak = peaks[peak_key(clk)]
    ach = flops / (ms / 1e3) / 1e12
    hbm = peaks['hbm_gbs']

    def gbs(nbytes, t_ms):
        v = nbytes / (t_ms / 1e3) / 1e9
        return {'ms': t_ms, 'gbs': v, 'hbm_frac': v / hbm}

    line = {
        'metric': 'grouped Muon optimizer step (3 ragged matrices per member)', 'value': 3 * P / (ms / 1e3),
        'unit': 'matrices/s', 'n_gpus': world, 'ms_per_step': ms, 'steps': args.steps, 'warmup': args.warmup,
        'higher_is_better': True, 'scaling': 'weak', 'dtype': 'bf16', 'data': 'synthetic',
        'config': {'workload': f'{P} members x 3 matrices, rows/cols U{{64..1024 step 16}}, 5 Newton-Schulz '
                               'iterations; AdamW on the 3 bias vectors' +
                               (f'; one replica per GPU' if world > 1 else ''),
                   'ns_tflop_per_step': flops / 1e12, 'elements': elems,
                   'newton_schulz': {'ms': ns_ms, 'tflops': flops / (ns_ms / 1e3) / 1e12,
                                     'frac': flops / (ns_ms / 1e3) / 1e12 / peak},
                   'muon_elementwise': dict(gbs(28.0 * elems, muon_el_ms), bytes_per_element=28),
                   'adamw_biases': dict(gbs(28.0 * adamw_elems, adamw_ms), elements=adamw_elems),
                   'adamw_weight_packs': dict(gbs(28.0 * big_elems, adamw_big_ms), elements=big_elems)},
        'roofline': {'bound': 'tensor', 'achieved': ach, 'peak': peak, 'unit': 'TFLOP/s', 'frac': ach / peak,
                     'peak_source': f'{kind} ({"sustained" if sustained else "burst"}: median SM clock '
                                    f'{clk["sm_mhz"]} of {clk["sm_max_mhz"]} MHz)',
                     'note': 'whole step (elementwise + Newton-Schulz) time against Newton-Schulz FLOPs'},
        'clocks': clk}
    if emit:
        print(json.dumps(line), flush=True)
    dist_done(emit)
    return line


def run_metrics(args) -> None:
    """Per-epoch evaluation of the full-training configuration's validation split: `members`
    binary-classification members x 100 000 rows.  Times the fused per-member BCE reduction,
    the per-member ROC AUC (sort-based) and the fused greedy ensemble selection (BCE, init top-1,
    at most 32 members), each as its own launch(es) with CUDA events; reports achieved GB/s
    against the measured HBM copy bandwidth."""
    import torch

    from tabpack_b200 import ops

    dev = torch.device('cuda', 0)
    torch.cuda.set_device(dev)
    P, N = args.members, 100_000
    g = torch.Generator(device=dev).manual_seed(7)
    y = (torch.rand(N, device=dev, generator=g) < 0.3).to(torch.int64)
    logits = torch.randn(P, N, device=dev, generator=g) + y.float() * torch.rand(P, 1, device=dev, generator=g) * 2
    proba = torch.sigmoid(logits)
    auc_ws = torch.empty(int(ops.load().tp_roc_auc_workspace_size(P, N, 0)), dtype=torch.uint8, device=dev)

    def timed(fn, reps):
        for _ in range(max(1, args.warmup)):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            out = fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / reps, out

    peaks, kind = load_peaks()
    with ClockSampler(0) as clocks:
        bce_ms, _ = timed(lambda: ops.metric_pack('bce', proba, y), args.steps)
        auc_ms, _ = timed(lambda: ops.binary_roc_auc(proba, y, auc_ws), max(1, args.steps // 4))
        greedy_ms, (counts, status) = timed(
            lambda: ops.greedy_ensemble(proba, y, metric='bce', maximize=False, max_ensemble_size=32),
            max(1, args.steps // 10))
    st = status.cpu().tolist()
    bce_bytes = 4.0 * P * N + 8.0 * N
    # the AUC sort moves each element's 4-byte key and 1-byte label: key build (read 4, write 5),
    # 4 radix passes (read 4 to count, read 5 + write 5 to scatter), one read of 5 for the ranks
    auc_bytes = P * N * (4.0 + 5.0 + 4 * 14.0 + 5.0)
    greedy_bytes = 4.0 * P * N * (st[0] + 1)  # every iteration scores all candidates once
    gbs = lambda b, ms: b / (ms / 1e3) / 1e9  # noqa: E731
    print(json.dumps({
        'metric': f'validation metrics + greedy ensemble ({P} members x {N} rows)',
        'value': bce_ms + auc_ms + greedy_ms, 'unit': 'ms', 'higher_is_better': False,
        'steps': args.steps, 'warmup': args.warmup,
        'config': {'workload': f'binary classification, {P} members x {N} validation rows, fp32 probabilities',
                   'bce': {'ms': bce_ms, 'gbs': gbs(bce_bytes, bce_ms), 'hbm_frac': gbs(bce_bytes, bce_ms) / peaks['hbm_gbs']},
                   'roc_auc': {'ms': auc_ms, 'gbs': gbs(auc_bytes, auc_ms),
                               'hbm_frac': gbs(auc_bytes, auc_ms) / peaks['hbm_gbs'],
                               'bytes_note': '70 B per element: key build (9) + 4 radix passes (14 each) + rank pass (5)'},
                   'greedy': {'ms': greedy_ms, 'iterations': st[0], 'members': st[1],
                              'gbs': gbs(greedy_bytes, greedy_ms), 'hbm_frac': gbs(greedy_bytes, greedy_ms) / peaks['hbm_gbs']},
                   'peak_source': f'{kind} (copy)'},
        'clocks': clocks.summary()}), flush=True)


# ----------------------------------------------------------------------------- full training

TRAIN_ROWS, VAL_ROWS, N_NUM, N_CAT, BATCH = 1_000_000, 100_000, 100, 10, 1024
STEPS_PER_EPOCH = -(-TRAIN_ROWS // BATCH)  # 977


def train_data(seed: int = 21):
    """The full-training configuration's synthetic data, identical on every rank: 1 000 000 train
    and 100 000 validation rows; 100 numerical features N(0, 1), 10 % of rows heavy-tailed
    (Student-t, 3 degrees of freedom); 10 categorical features with cardinalities log-U[2, 1000];
    labels Bernoulli(sigmoid(random teacher MLP)).  Drawn on the host from fixed seeds."""
    import torch

    cards = train_cards(seed)
    n = TRAIN_ROWS + VAL_ROWS
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(n, N_NUM, generator=g)
    heavy = torch.rand(n, generator=g) < 0.1
    # Student-t(3) = N(0, 1) / sqrt(chi2(3) / 3)
    z = torch.randn(int(heavy.sum()), N_NUM, generator=g)
    chi2 = torch.randn(int(heavy.sum()), N_NUM, 3, generator=g).square().sum(-1)
    x[heavy] = z / torch.sqrt(chi2 / 3)
    xc = torch.stack([torch.randint(0, c, (n,), generator=g) for c in cards], 1)
    w1 = torch.randn(N_NUM, 64, generator=g) / N_NUM ** 0.5
    w2 = torch.randn(64, generator=g) / 8
    y = (torch.rand(n, generator=g) < torch.sigmoid(torch.relu(x @ w1) @ w2 - 0.5)).to(torch.int64)
    split = {'train': slice(0, TRAIN_ROWS), 'val': slice(TRAIN_ROWS, n)}
    return cards, {k: {'x_num': x[s], 'x_cat': xc[s], 'y': y[s]} for k, s in split.items()}


def train_cards(seed: int = 21) -> list[int]:
    """Cardinalities of the 10 categorical features, log-U[2, 1000]."""
    rng = np.random.default_rng(seed)
    return [int(c) for c in np.exp(rng.uniform(np.log(2), np.log(1000), N_CAT)).round()]


def train_members(n: int, seed: int = 21) -> list[dict]:
    """Per-member hyperparameters of the full-training pack: depth U{1..4}, width U{128..1024
    step 8}, dropout U[0, 0.5]."""
    rng = np.random.default_rng(seed + 1)
    return [dict(n_blocks=int(rng.integers(1, 5)), d_block=int(rng.integers(16, 129)) * 8,
                 dropout=float(rng.uniform(0, 0.5))) for _ in range(n)]


def train_work(per: list[dict], d_in: int, batch: int = BATCH) -> dict[str, float]:
    """Algorithmic FLOPs per training step by kernel family (ragged shapes, active blocks only):
    forward / dgrad / wgrad GEMMs of the blocks and the 1-wide head (the first layer takes no
    input gradient), and the Newton-Schulz GEMMs of Muon (5 iterations of 4 r^2 c + 2 r^3 per
    block weight, r = min and c = max of its shape)."""
    fwd = dgrad = wgrad = ns = ns_exec = 0.0
    for pm in per:
        w, nb = pm['d_block'], pm['n_blocks']
        mm = d_in * w + (nb - 1) * w * w + w
        fwd += 2.0 * batch * mm
        wgrad += 2.0 * batch * mm
        dgrad += 2.0 * batch * ((nb - 1) * w * w + w)
        for j in range(nb):
            r, c = min(w, d_in if j == 0 else w), max(w, d_in if j == 0 else w)
            ns += 5.0 * (4.0 * r * r * c + 2.0 * r ** 3)
            ns_exec += 5.0 * (2.0 * r * r * c * ns_symmetric_fraction(r) + 2.0 * r ** 3 * ns_symmetric_fraction(r)
                              + 2.0 * r * r * c)
    return {'fwd': fwd, 'dgrad': dgrad, 'wgrad': wgrad, 'newton_schulz': ns, 'newton_schulz_executed': ns_exec}


def ns_symmetric_fraction(r: int) -> float:
    """Fraction of an r x r symmetric Newton-Schulz product (A = X X^T, B = b A + c A^2) that
    the kernels compute directly: the 128 x 256 tiles not entirely below the diagonal (the rest
    are written as transposes), counted over the matrix's r x r elements."""
    done = 0
    for nt in range((r + 255) // 256):
        cols = min(256, r - 256 * nt)
        for mt in range(min((r + 127) // 128, 2 * nt + 2)):
            done += min(128, r - 128 * mt) * cols
    return done / float(r * r)


def member_cost(pm: dict, d_in: int) -> float:
    """A member's estimated device time per training step (the sharding weight): its tensor-core
    FLOPs as the kernels execute them at ~800 TFLOP/s plus the bytes its weights move through
    the Muon elementwise kernels and the bf16 copies (~30 B per weight element) at ~5 TB/s."""
    w = train_work([pm], d_in)
    flops = w['fwd'] + w['dgrad'] + w['wgrad'] + w['newton_schulz_executed']
    wd = pm['d_block']
    elements = d_in * wd + (pm['n_blocks'] - 1) * wd * wd
    return flops / 800e12 + 30.0 * elements / 5e12


def _compact(line: dict) -> dict:
    """The figures of another workload's JSON line that the training line carries."""
    keep = ('workload', 'per_kernel_ms', 'ragged_tflop_per_step_per_gpu', 'ragged_tflops_achieved',
            'ns_tflop_per_step', 'newton_schulz', 'muon_elementwise', 'adamw_biases', 'adamw_weight_packs',
            'member_rows_per_s', 'ragged_tflops', 'frac_of_sustained_bf16', 'head_checksum')
    out = {k: line[k] for k in ('metric', 'value', 'unit', 'ms_per_step', 'steps', 'warmup', 'scaling')
           if k in line}
    out['config'] = {k: v for k, v in line.get('config', {}).items() if k in keep}
    for k in ('roofline', 'e2e', 'clocks'):
        if line.get(k) is not None:
            out[k] = line[k]
    return out


def run_other_configs(args) -> dict:
    """The other benchmark configurations, measured after the training region in the same run
    (every rank takes part; short step counts): the ragged GEMM layer (256 members per GPU), the
    grouped optimizer step (1024 members, one replica per GPU) and packed inference (1024
    members over all GPUs, all-reduced ensemble head).  Returns compact results (rank 0)."""
    import torch

    global MEMBERS
    out = {}
    runs = (('ragged_gemm_layer', run_b200, 256, 50, 5), ('grouped_optimizer', run_optimizer, 1024, 5, 2),
            ('packed_inference', run_inference, 1024, 3, 1))
    saved = MEMBERS
    for name, fn, members, steps, warmup in runs:
        sub = argparse.Namespace(**vars(args))
        sub.members, sub.steps, sub.warmup, sub.no_cpu_baseline = members, steps, warmup, True
        MEMBERS = members
        try:
            line = fn(sub, emit=False)
        finally:
            MEMBERS = saved
        torch.cuda.empty_cache()
        if line is not None:
            out[name] = _compact(line)
    return out


def run_train(args) -> None:
    """Full TabPack training of the full-training configuration, members sharded over the GPUs.

    The global pack (512 members by default) is split into contiguous member ranges balanced by
    FLOPs per step (strong scaling: the pack is fixed, each rank trains its share).  The timed
    region is an epoch scaled down to K steps: K training steps (batch gather, one-hot first-layer
    input, forward, BCE loss, backward, Muon + AdamW) over the first K x 1024 training rows, then
    the epoch end over the first K / 977 of the validation rows -- every member's predictions,
    all-gathered over NCCL, and a greedy ensemble built from them -- so training and evaluation
    stand in the same ratio as in a full epoch.  value = member-samples/s of the whole job."""
    import datetime

    import torch
    import torch.distributed as dist

    from tabpack_b200 import ops
    from tabpack_b200.training import OnlineEnsemble, PackTrainer

    world = int(os.environ.get('WORLD_SIZE', '1'))
    rank = int(os.environ.get('RANK', '0'))
    local = int(os.environ.get('LOCAL_RANK', '0'))
    torch.cuda.set_device(local)
    dev = torch.device('cuda', local)
    if world > 1:
        dist.init_process_group('nccl', device_id=dev, timeout=datetime.timedelta(seconds=300))
    P, K, W = args.members, args.steps, args.warmup
    cards, data = train_data()
    d_in = N_NUM + sum(cards)
    per = train_members(P)
    if args.embeddings == 'cosine':
        rng = np.random.default_rng(23)
        for pm in per:
            pm['numerical_embeddings'] = {'d_embedding': int(rng.integers(8, 33)),
                                          'init_scale': float(np.exp(rng.uniform(np.log(0.01), np.log(1.0))))}
    model = dict(n_numerical_features=N_NUM, categorical_cardinalities=cards, d_out=1, max_d_block=1024,
                 max_n_blocks=4)
    if args.embeddings == 'cosine':
        from tabpack_b200.nn import CosineEmbeddingsPack

        model['numerical_embeddings'] = {'type': CosineEmbeddingsPack, 'max_d_embedding': 32}
    trainer = PackTrainer(n_members=P, model=model, per_member_model=per,
                          optimizer=dict(type='muon', adamw_lr=1e-3, weight_decay=1e-5, muon_lr=2e-2), loss='bce',
                          seed=0, device=dev, autocast_bf16=True, cost=[member_cost(pm, d_in) for pm in per])
    val_rows = min(VAL_ROWS, (math.ceil(VAL_ROWS * K / STEPS_PER_EPOCH) + 255) // 256 * 256)
    host = {'train': {k: v[: K * BATCH] for k, v in data['train'].items()},
            'val': {k: v[:val_rows] for k, v in data['val'].items()}}
    dev_data = {s: {k: v.to(dev) for k, v in d.items()} for s, d in host.items()}
    warm = {k: v.to(dev) for k, v in (
        (k, data['train'][k][K * BATCH: (K + max(W, 1)) * BATCH]) for k in data['train'])}
    del data

    def epoch(train, val, ep, on_step=None):
        loss = trainer.fit_epoch(train, batch_size=BATCH, epoch=ep, on_step=on_step)
        preds = trainer.predict(val)  # (P_total, rows), all-gathered over NCCL
        ens = OnlineEnsemble(trainer._score(val['y']))
        ens.update(lambda key: preds[key[0]], [], [(g, K) for g in trainer.gathered_ids])
        return loss, preds, ens

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])
        torch.cuda.synchronize()

    torch.autograd.set_multithreading_enabled(False)  # backward launches from the calling thread
    epoch(warm, dev_data['val'], 0)  # warm-up: W steps and one epoch end
    barrier()
    stream = torch.cuda.current_stream(dev)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
    with ClockSampler(local) as clocks:
        torch.cuda.nvtx.range_push('timed')  # lets a profiler keep only the timed region
        ev[0].record(stream)
        loss = trainer.fit_epoch(dev_data['train'], batch_size=BATCH, epoch=1)
        ev[1].record(stream)
        preds = trainer.predict(dev_data['val'])
        ens = OnlineEnsemble(trainer._score(dev_data['val']['y']))
        ens.update(lambda key: preds[key[0]], [], [(g, K) for g in trainer.gathered_ids])
        ev[2].record(stream)
        torch.cuda.nvtx.range_pop()
        barrier()
    region_ms, train_ms = ev[0].elapsed_time(ev[2]), ev[0].elapsed_time(ev[1])

    # end to end through the same public calls: the step inputs (the epoch's training and
    # validation rows) copied from pinned host memory inside the region, each step's
    # per-member losses and the gathered validation predictions read back to the host
    pinned = {s: {k: v.pin_memory() for k, v in d.items()} for s, d in host.items()}
    loss_host = torch.empty(K, trainer.hi - trainer.lo).pin_memory()
    pred_host = torch.empty(P, val_rows).pin_memory()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    up = {s: {k: v.to(dev, non_blocking=True) for k, v in d.items()} for s, d in pinned.items()}
    _, preds_e2e, _ = epoch(up['train'], up['val'], 2,
                            on_step=lambda i, l: loss_host[i].copy_(l, non_blocking=True))
    pred_host.copy_(preds_e2e, non_blocking=True)
    e1.record(stream)
    barrier()
    e2e_ms = e0.elapsed_time(e1)

    # per-family kernel time over one more scaled epoch, launch by launch (CUDA events on the
    # one stream every launch of the step runs on)
    with ops.KernelTimes() as kt:
        epoch(dev_data['train'], dev_data['val'], 3)
    barrier()

    t = torch.tensor([region_ms, train_ms, e2e_ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    region_ms, train_ms, e2e_ms = (float(v) for v in t)
    # shard-invariance checksum: the trained pack's gathered validation predictions
    final = trainer.predict(dev_data['val']).float().cpu().numpy()
    import hashlib

    checksum = {'sha256_16': hashlib.sha256(final.tobytes()).hexdigest()[:16], 'sum': float(final.astype(np.float64).sum())}
    local_work = train_work(per[trainer.lo: trainer.hi], d_in)
    members_per_rank = [b - a for a, b in trainer.ranges]
    local_members = trainer.hi - trainer.lo
    fam_ms = {k: kt.ms[k] / K for k in kt.ms if kt.launches[k]}
    fam_ms['newton_schulz'] = fam_ms.pop('newton_schulz_gram', 0.0) + fam_ms.pop('newton_schulz_update', 0.0)
    ns_exec = local_work.pop('newton_schulz_executed')
    mean_loss = float(loss.mean())
    del trainer, dev_data, pinned, up, warm, preds, preds_e2e, ens, loss
    torch.cuda.empty_cache()
    other = {} if args.no_other_configs else run_other_configs(args)
    if world > 1:
        dist.destroy_process_group()
    if rank != 0:
        return

    peaks, peak_kind = load_peaks()
    clk = clocks.summary()
    sustained = peak_key(clk) == 'bf16_tflops_sustained'
    peak = peaks[peak_key(clk)]
    gemm = {}
    for fam in ('fwd', 'dgrad', 'wgrad', 'newton_schulz'):
        if fam_ms.get(fam):
            ach = local_work[fam] / (fam_ms[fam] / 1e3) / 1e12
            gemm[fam] = {'ms_per_step': fam_ms[fam], 'tflop_per_step': local_work[fam] / 1e12, 'tflops': ach,
                         'frac': ach / peak}
    if 'newton_schulz' in gemm:
        # the symmetric products compute only the tiles on or above the diagonal: the FLOPs
        # the kernels execute, beside the reference iteration's algorithmic count above
        ex = ns_exec / (fam_ms['newton_schulz'] / 1e3) / 1e12
        gemm['newton_schulz'].update({'executed_tflop_per_step': ns_exec / 1e12, 'executed_tflops': ex,
                                      'executed_frac': ex / peak})
    dominant = max(gemm, key=lambda f: gemm[f]['ms_per_step'])
    roof = {'bound': 'tensor', 'achieved': gemm[dominant]['tflops'], 'peak': peak, 'unit': 'TFLOP/s',
            'frac': gemm[dominant]['frac'], 'kernel': dominant,
            'traffic': (TRAIN_TRAFFIC_BYTES_PER_MEMBER_STEP[dominant] * local_members
                        if dominant in TRAIN_TRAFFIC_BYTES_PER_MEMBER_STEP else None),
            'traffic_per': 'step (all launches of the family on this rank)',
            'peak_source': f'{peak_kind} ({"sustained" if sustained else "burst"}: median SM clock '
                           f'{clk["sm_mhz"]} of {clk["sm_max_mhz"]} MHz in the region)'}
    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        cpu, _ = train_cpu_sample(cards, per, budget_s=args.cpu_seconds)
    samples = P * BATCH * K
    launches = sum(kt.launches.values())
    line = {
        'metric': 'member-samples/sec train (full TabPack training, Muon + AdamW)', 'value': samples / (region_ms / 1e3),
        'unit': 'member-samples/s', 'n_gpus': world, 'steps': K, 'warmup': W, 'ms_per_step': region_ms / K,
        'higher_is_better': True, 'scaling': 'strong', 'vs_baseline': None, 'dtype': 'bf16', 'data': 'synthetic',
        'config': {'workload': f'full TabPack training: {P} members (depth U{{1..4}}, width U{{128..1024}}, '
                               f'dropout U[0,0.5]), {N_NUM} numerical + {N_CAT} categorical features '
                               f'({sum(cards)} one-hot columns), batch {BATCH}, BCE, Muon + AdamW, bf16; '
                               f'timed: {K} steps + the epoch end over {val_rows} validation rows (all-gather + '
                               f'greedy ensemble)' + (', cosine numerical embeddings' if args.embeddings == 'cosine'
                                                      else ''),
                   'members': P, 'members_per_rank': members_per_rank,
                   'parallelism': f'member-sharded x{world} (ranges balanced by FLOPs per step)',
                   'train_ms_per_step': train_ms / K, 'epoch_end_ms': region_ms - train_ms,
                   'l2': 'weights and optimizer state exceed L2 (about 40 GB at 512 members)',
                   'per_kernel_ms_per_step': fam_ms, 'gemm': gemm, 'checksum': checksum,
                   'mean_train_loss': mean_loss, 'other_configs': other},
        'roofline': roof,
        'cpu_baseline': cpu,
        'e2e': {'value': samples / (e2e_ms / 1e3), 'unit': 'member-samples/s',
                'h2d_bytes_per_step': sum(v.numel() * v.element_size() for d in host.values() for v in d.values()) / K,
                'd2h_bytes_per_step': loss_host.numel() * 4 / K + pred_host.numel() * 4 / K},
        'gpu_launches': launches,
        'clocks': clk,
    }
    print(json.dumps(line), flush=True)


# DRAM bytes (read + write) per training step and member of a kernel family, from an ncu
# capture of the training workload's launches at 64 members (the 15 Newton-Schulz launches of
# one step: 7.528 GB, `dram__bytes_read.sum + dram__bytes_write.sum`), scaled by the members a
# rank trains.
TRAIN_TRAFFIC_BYTES_PER_MEMBER_STEP: dict[str, float] = {'newton_schulz': 7.528e9 / 64}


def train_cpu_sample(cards: list[int], per: list[dict], *, budget_s: float, steps: int | None = None,
                     members: int = 16):
    """The reference's training step on the host (`oracle.torch_step`, all host threads) on the
    first `members` members of the pack; returns the cpu_baseline dict and the per-step values."""
    import torch

    from oracle.torch_step import TrainingStep, sample_batch

    torch.set_num_threads(os.cpu_count() or 1)
    sub = per[:members]
    step = TrainingStep(n_num=N_NUM, cards=cards, widths=[p['d_block'] for p in sub],
                        depths=[p['n_blocks'] for p in sub], dropout=[p['dropout'] for p in sub])
    rng = np.random.default_rng(5)
    g = torch.Generator().manual_seed(5)
    n = 65536
    x = torch.randn(n, N_NUM, generator=g)
    xc = torch.stack([torch.randint(0, c, (n,), generator=g) for c in cards], 1)
    y = (torch.rand(n, generator=g) < 0.3).to(torch.int64)
    step.step(*sample_batch(rng, x, xc, y, members, BATCH))  # warm-up
    vals, t_all = [], time.perf_counter()
    while True:
        b = sample_batch(rng, x, xc, y, members, BATCH)
        t0 = time.perf_counter()
        step.step(*b)
        vals.append(members * BATCH / (time.perf_counter() - t0))
        if (steps is not None and len(vals) >= steps) or (steps is None and time.perf_counter() - t_all >= budget_s):
            break
    return {'value': statistics.median(vals), 'unit': 'member-samples/s', 'cores': torch.get_num_threads(),
            'kind': 'port', 'sample': f'the first {members} members of the pack, batch {BATCH}, {len(vals)} training '
                                      'steps (torch CPU restatement of the reference step: padded baddbmm, '
                                      'bernoulli_ dropout, BCE, autograd, Muon with bf16 Newton-Schulz + AdamW, '
                                      'bf16 autocast)'}, vals


def run_train_reference(args) -> None:
    """The reference arm of the full-training workload: its CPU step on the host cores (rank 0
    only; other ranks exit), K timed steps of a 16-member sample after W warm-up steps."""
    if int(os.environ.get('RANK', '0')) != 0:
        return
    cards = train_cards()
    per = train_members(args.members)
    cpu, vals = train_cpu_sample(cards, per, budget_s=0.0, steps=args.warmup + args.steps)
    vals = vals[args.warmup:]
    value = statistics.median(vals)
    cpu['value'] = value
    cpu['sample'] = cpu['sample'].replace(f'{args.warmup + args.steps} training steps',
                                          f'{args.steps} timed training steps after {args.warmup}')
    line = {
        'metric': 'member-samples/sec train (full TabPack training, Muon + AdamW)', 'value': value,
        'unit': 'member-samples/s', 'n_gpus': args.gpus, 'steps': args.steps, 'warmup': args.warmup,
        'ms_per_step': 16 * BATCH / value * 1e3, 'higher_is_better': True, 'scaling': 'strong',
        'vs_baseline': None, 'dtype': 'bf16', 'data': 'synthetic', 'impl': 'reference',
        'config': {'workload': 'full TabPack training (the pack of the default workload), reference step on the '
                               'host cores', 'sample_members': 16},
        'cpu_baseline': cpu,
        'e2e': {'value': value, 'unit': 'member-samples/s', 'h2d_bytes_per_step': 0, 'd2h_bytes_per_step': 0},
    }
    print(json.dumps(line), flush=True)


def run_inference(args, emit: bool = True) -> dict | None:
    """Inference of the packed-ensemble inference configuration: `members` members over all
    ranks (1024 by default; rank r predicts its share), depth U{2,3}, width U{256..1024 step
    8}, 200 numerical features N(0, 1), a 10-class head, batches of 65 536 rows in bf16.  A step
    is every member's class probabilities for one batch (members run in groups of 128) and the
    ensemble head, the mean of 64 seeded members' probabilities, summed over ranks with an
    NCCL all-reduce.  value = rows/s (strong scaling: the pack is fixed); e2e copies each
    batch from pinned host memory and reads the ensemble head back."""
    import datetime

    import torch
    import torch.distributed as dist

    from tabpack_b200.training import PackPredictor, PackTrainer

    rank = int(os.environ.get('RANK', '0'))
    local = int(os.environ.get('LOCAL_RANK', '0'))
    torch.cuda.set_device(local)
    dev = torch.device('cuda', local)
    world = dist_init(dev)
    total, B, n_num, C = args.members, 65536, 200, 10
    rng = np.random.default_rng(31)
    per = [dict(n_blocks=int(rng.integers(2, 4)), d_block=int(rng.integers(32, 129)) * 8, dropout=0.0)
           for _ in range(total)]
    model = dict(n_numerical_features=n_num, categorical_cardinalities=[], d_out=C, max_d_block=1024, max_n_blocks=3)
    trainer = PackTrainer(n_members=total, model=model, per_member_model=per,
                          optimizer=dict(type='adamw', lr=1e-3, weight_decay=0.0), loss='ce', seed=0, device=dev,
                          autocast_bf16=True)
    ens = torch.from_numpy(np.random.default_rng(7).choice(total, 64, replace=False)).to(dev)
    predictor = PackPredictor(trainer, {'ensemble': ens})
    # ragged GEMM FLOPs per row of this rank's members (first layer, hidden blocks, head)
    flops_row = 0.0
    for pm in per[trainer.lo: trainer.hi]:
        w = pm['d_block']
        flops_row += 2.0 * (n_num * w + (pm['n_blocks'] - 1) * w * w + w * C)
    g = torch.Generator(device=dev).manual_seed(11 + rank)
    x = torch.randn(B, n_num, device=dev, generator=g)
    x_host = x.cpu().pin_memory()
    chunk = 128

    def step():
        return predictor(x, None, eval_batch_size=B, member_chunk=chunk)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        step()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        e0.record()
        for _ in range(args.steps):
            step()
        e1.record()
        barrier()
    ms = e0.elapsed_time(e1) / args.steps
    # end to end: batch from pinned host memory, ensemble head back to the host
    xd = torch.empty_like(x)
    barrier()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(args.steps):
        xd.copy_(x_host, non_blocking=True)
        _, heads = predictor(xd, None, eval_batch_size=B, member_chunk=chunk)
        head = heads['ensemble'].cpu()
    t1.record()
    barrier()
    e2e_ms = t0.elapsed_time(t1) / args.steps
    t = torch.tensor([ms, e2e_ms], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, e2e_ms = float(t[0]), float(t[1])
    flops = torch.tensor([flops_row * B], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(flops)
    peaks, kind = load_peaks()
    tflops = float(flops[0]) / (ms / 1e3) / 1e12
    line = None
    if rank == 0:
        line = {
            'metric': 'rows/sec inference (every member of the pack, ensemble head)', 'value': B / (ms / 1e3),
            'unit': 'rows/s', 'n_gpus': world, 'steps': args.steps, 'warmup': args.warmup, 'ms_per_step': ms,
            'higher_is_better': True, 'scaling': 'strong', 'vs_baseline': None, 'dtype': 'bf16', 'data': 'synthetic',
            'config': {'workload': f'{total} members, depth U{{2,3}}, width U{{256..1024}}, 200 numerical features, '
                                   f'10 classes, batch {B} rows, ensemble of 64 members, members in groups of {chunk}',
                       'member_rows_per_s': total * B / (ms / 1e3), 'ragged_tflops': tflops,
                       'frac_of_sustained_bf16': tflops / peaks['bf16_tflops_sustained'], 'peak_source': kind,
                       'head_checksum': float(head.double().sum())},
            'e2e': {'value': B / (e2e_ms / 1e3), 'unit': 'rows/s', 'h2d_bytes_per_step': x.numel() * 4,
                    'd2h_bytes_per_step': B * C * 4},
            'clocks': clocks.summary()}
        if emit:
            print(json.dumps(line), flush=True)
    del trainer, predictor
    dist_done(emit)
    return line


def run_onehot(args) -> None:
    """The first layer of the full-training configuration over one-hot categoricals, piece by
    piece, gathered against dense: `members` members, batch 1024 gathered from 1 000 000 rows,
    100 numerical features, 10 categorical features with cardinalities log-U[2, 1000] (the
    full-training draw), output widths U{128..1024 step 8}, bf16, ReLU and dropout
    p ~ U[0, 0.5].  Each piece: median of `steps` CUDA-event timings after `warmup` calls.
    value = the gathered forward (category sort, gather, dense-column GEMM with the addend)."""
    import statistics

    import torch

    from tabpack_b200 import ops

    dev = torch.device('cuda', 0)
    torch.cuda.set_device(dev)
    P, B, n_num, N, max_out = args.members, 1024, 100, 1_000_000, 1024
    rng = np.random.default_rng(21)
    cards = [int(c) for c in np.exp(rng.uniform(np.log(2), np.log(1000), 10)).round()]
    offs = torch.tensor([0] + list(np.cumsum(cards)), dtype=torch.int32, device=dev)
    n_oh = int(offs[-1])
    d_in = n_num + n_oh
    outs = torch.from_numpy(rng.integers(16, 129, P).astype(np.int32) * 8).to(dev)
    g = torch.Generator(device=dev).manual_seed(0)
    W = torch.randn(P, max_out, d_in, device=dev, generator=g) * 0.02
    b = torch.zeros(P, max_out, device=dev)
    xn = torch.randn(N, n_num, device=dev, generator=g)
    xc = torch.stack([torch.randint(0, c, (N,), device=dev, generator=g) for c in cards], 1)
    idx = torch.randint(0, N, (P, B), device=dev, generator=g)
    p = torch.rand(P, device=dev, generator=g) * 0.5
    dense_cols, full_cols = (n_num + 7) // 8 * 8, (d_in + 7) // 8 * 8
    wd = torch.zeros(P, max_out, dense_cols, dtype=torch.bfloat16, device=dev)
    wt = torch.empty(P, n_oh, max_out, dtype=torch.bfloat16, device=dev)
    wf = torch.zeros(P, max_out, full_cols, dtype=torch.bfloat16, device=dev)
    kw = dict(out_features=outs, relu=True, dropout_p=p, seed=3, offset=1)
    res = {}

    def timed(name, fn):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        ts = []
        for _ in range(args.steps):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            torch.cuda.synchronize()
            ts.append(e0.elapsed_time(e1))
        res[name] = statistics.median(ts)

    with ClockSampler(0) as clocks:
        timed('cast_dense_columns', lambda: ops.weight_cast(W, wd, out_features=outs, src_cols=n_num))
        timed('cast_onehot_transposed', lambda: ops.weight_cast_transposed(W, wt, col0=n_num, ncols=n_oh,
                                                                           out_features=outs))
        timed('cast_whole_weight', lambda: ops.weight_cast(W, wf, out_features=outs))
        timed('input_dense', lambda: ops.tabpack_input(xn, None, offs, dense_cols, torch.bfloat16, row_index=idx))
        timed('input_with_onehot', lambda: ops.tabpack_input(xn, xc, offs, full_cols, torch.bfloat16, row_index=idx))
        xd = ops.tabpack_input(xn, None, offs, dense_cols, torch.bfloat16, row_index=idx)
        xf = ops.tabpack_input(xn, xc, offs, full_cols, torch.bfloat16, row_index=idx)
        out = {}
        timed('gathered_forward', lambda: out.__setitem__('g', ops.onehot_linear_forward(
            xd, wd, b, x_cat=xc, cat_offsets=offs, n_dense=n_num, w_onehot_t=wt, row_index=idx, **kw)))
        timed('dense_forward', lambda: out.__setitem__('d', ops.linear_forward(xf, wf, b, **kw)))
        (yg, st), yd = out['g'], out['d']
        dy = torch.randn(P, B, max_out, device=dev, generator=g).bfloat16()
        timed('gathered_backward', lambda: ops.onehot_linear_backward(dy, xd, wd, yg, st, **kw, dw_rows=max_out,
                                                                      db_cols=max_out))
        timed('dense_backward', lambda: ops.linear_backward(dy, xf, wf, yd, **kw, need_dx=False,
                                                            dw_shape=(max_out, d_in), db_cols=max_out))
    diff = float((yg.float() - yd.float()).abs().max() / yd.float().abs().max())
    print(json.dumps({
        'metric': 'first-layer forward over one-hot categoricals (gathered)', 'value': res['gathered_forward'],
        'unit': 'ms', 'higher_is_better': False, 'steps': args.steps, 'warmup': args.warmup, 'dtype': 'bf16',
        'data': 'synthetic',
        'config': {'workload': f'{P} members, batch {B} gathered from {N} rows, {n_num} numerical + 10 categorical '
                               f'features ({n_oh} one-hot columns), widths U{{128..1024}}, ReLU + dropout',
                   'ms': res, 'gathered_vs_dense_max_rel_diff': diff},
        'clocks': clocks.summary()}), flush=True)


def main() -> None:
    global MEMBERS
    ap = argparse.ArgumentParser()
    ap.add_argument('--gpus', type=int, default=1)
    ap.add_argument('--steps', type=int, default=None, help='timed steps (default 20; 300 for the layer workload)')
    ap.add_argument('--warmup', type=int, default=None, help='warm-up steps (default 5; 10 for the layer workload)')
    ap.add_argument('--impl', choices=['b200', 'reference'], default='b200')
    ap.add_argument('--cpu-seconds', type=float, default=15.0)
    ap.add_argument('--no-cpu-baseline', action='store_true')
    ap.add_argument('--members', type=int, default=None,
                    help='members: of the whole pack for train (512) and inference (1024), per GPU for the layer '
                         'workload (256), of the optimizer (1024), metrics (512) and onehot (512) workloads')
    ap.add_argument('--workload', choices=['train', 'layer', 'optimizer', 'metrics', 'inference', 'onehot'],
                    default='train',
                    help='train: full TabPack training steps and the epoch end, members sharded over the GPUs '
                         '(default); layer: one packed MLP block forward+backward; optimizer: grouped Muon step; '
                         'metrics: validation metrics, ROC AUC and greedy selection; inference: packed predictor; '
                         'onehot: the one-hot first layer piece by piece')
    ap.add_argument('--no-other-configs', action='store_true',
                    help='train workload: skip the other configurations measured after the training region')
    ap.add_argument('--embeddings', choices=['none', 'cosine'], default='none',
                    help='train workload: numerical features raw or through cosine embeddings')
    args = ap.parse_args()
    if args.members is None:
        args.members = {'optimizer': 1024, 'metrics': 512, 'train': 512, 'inference': 1024,
                        'onehot': 512}.get(args.workload, MEMBERS)
    if args.steps is None:
        args.steps = 300 if args.workload == 'layer' else 20
    if args.warmup is None:
        args.warmup = 10 if args.workload == 'layer' else 5
    MEMBERS = args.members
    if args.impl == 'reference':
        if args.workload == 'train':
            run_train_reference(args)
        elif args.workload == 'layer':
            run_reference(args)
        elif int(os.environ.get('RANK', '0')) == 0:
            print(json.dumps({'impl': 'reference', 'unavailable': f'no CPU reference arm for the {args.workload} '
                                                                  'workload (train and layer have one)'}), flush=True)
        return
    {'train': run_train, 'layer': run_b200, 'optimizer': run_optimizer, 'metrics': run_metrics,
     'inference': run_inference, 'onehot': run_onehot}[args.workload](args)


if __name__ == '__main__':
    main()
