"""Benchmark of the packed-ensemble hot path on B200: the ragged grouped GEMM layer.

Workload (per GPU): a pack of 256 members sharing one 4096 x 512 bf16 input
batch; member i has its own output width out_i ~ U{64, 80, ..., 1024}, weights
U(+-1/sqrt(512)), a bias, ReLU and dropout with p_i ~ U[0, 0.5].  One step is
the forward pass (one fused launch: GEMM + bias + ReLU + Philox dropout) and the
backward pass (activation/bias gradient, dgrad, wgrad) of that layer, i.e.
3 x sum_i 2 * 4096 * 512 * out_i ragged FLOPs.  Members are sharded over GPUs
(weak scaling: every rank owns its own 256 members, keyed by global member id);
the layer has no cross-member exchange, so the timed region has no collective.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

Prints one JSON line (rank 0).  `value` is whole-job member-samples/s with all
inputs resident in HBM; `e2e` repeats the measurement through the same C-ABI
calls with the input batch copied from pinned host memory and the bias
gradient read back every step; `roofline` covers the kernel with the largest
share of the step; `cpu_baseline` times the numpy restatement of the same layer
on a bounded member sample on this host.  `--impl reference` times that CPU
restatement alone, with all host threads.
"""

from __future__ import annotations

import argparse
import ctypes
import json
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
            'out widths U{64..1024 step 16}, bias + ReLU + Philox dropout p~U[0,0.5], fp32 accumulation')


def member_widths(base: int, n: int) -> np.ndarray:
    """Per-member output widths, seeded by global member id (shard-invariant)."""
    out = np.empty(n, np.int32)
    for i in range(n):
        out[i] = np.random.default_rng(1_000_003 * (base + i) + 7).integers(4, 65) * 16
    return out


def member_dropout(base: int, n: int) -> np.ndarray:
    return np.array([np.random.default_rng(7_000_001 * (base + i) + 3).uniform(0, 0.5) for i in range(n)], np.float32)


def load_peaks() -> tuple[dict, str]:
    path = os.path.join(ROOT, 'MEASURED_PEAKS.json')
    if os.path.exists(path):
        with open(path) as f:
            return json.load(f), 'measured'
    return {'hbm_gbs': 6650.0, 'bf16_tflops': 1590.0, 'bf16_tflops_sustained': 1400.0}, 'fallback'


# ----------------------------------------------------------------------------- CPU legs


def cpu_layer_step(x, w, b, out_f, p, dy, seed, offset):
    """numpy restatement (oracle) of one forward+backward of the layer."""
    from oracle import layers as ol

    P = w.shape[0]
    mv = ol.dropout_mask_values(seed=seed, offset=offset, members=np.arange(P), n_rows=x.shape[0],
                                n_cols=w.shape[1], p=p, dtype=np.float32)
    y, pre = ol.block_forward(x, w, b, out_f, mask_values=mv)
    ol.block_backward(x, w, out_f, pre, dy, mask_values=mv)
    return y


def cpu_sample(members: int, budget_s: float, steps: int | None = None):
    """Times the CPU restatement on `members` members; returns (member-samples/s, threads, sample)."""
    rng = np.random.default_rng(0)
    out_f = member_widths(0, members)
    max_out = int(out_f.max())
    x = rng.standard_normal((ROWS, D_IN)).astype(np.float32)
    w = (rng.uniform(-1, 1, (members, max_out, D_IN)) / np.sqrt(D_IN)).astype(np.float32)
    b = (rng.uniform(-1, 1, (members, max_out)) / np.sqrt(D_IN)).astype(np.float32)
    p = member_dropout(0, members)
    dy = rng.standard_normal((members, ROWS, max_out)).astype(np.float32)
    cpu_layer_step(x, w, b, out_f, p, dy, 1, 0)  # warm-up
    n, t0 = 0, time.perf_counter()
    while True:
        cpu_layer_step(x, w, b, out_f, p, dy, 1, n + 1)
        n += 1
        el = time.perf_counter() - t0
        if (steps is not None and n >= steps) or (steps is None and el >= budget_s):
            break
    try:
        from threadpoolctl import threadpool_info

        threads = max([i.get('num_threads', 1) for i in threadpool_info()] or [1])
    except Exception:  # pragma: no cover
        threads = os.cpu_count() or 1
    sample = f'{members} members x {ROWS} rows x {D_IN} in (out widths {int(out_f.sum())} total), {n} fwd+bwd steps'
    return members * ROWS * n / el, threads, sample


def run_reference(args) -> None:
    rank = int(os.environ.get('RANK', '0'))
    if rank != 0:
        return
    members = 4
    vals = []
    threads = 1
    sample = ''
    for _ in range(max(args.warmup, 0)):
        cpu_sample(members, 0, steps=1)
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
                         'sample': sample + ' per step (numpy restatement of the reference layer)'},
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


def run_b200(args) -> None:
    import torch
    import torch.distributed as dist

    from tabpack_b200 import _lib

    world = int(os.environ.get('WORLD_SIZE', '1'))
    rank = int(os.environ.get('RANK', '0'))
    local = int(os.environ.get('LOCAL_RANK', '0'))
    torch.cuda.set_device(local)
    dev = torch.device('cuda', local)
    if world > 1:
        import datetime

        dist.init_process_group('nccl', device_id=dev, timeout=datetime.timedelta(seconds=120))
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
    y = torch.empty(MEMBERS, ROWS, MAX_OUT, device=dev, dtype=torch.bfloat16)
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
        roof = {'bound': 'tensor', 'achieved': ach, 'peak': peaks['bf16_tflops_sustained'], 'unit': 'TFLOP/s'}
    roof['frac'] = roof['achieved'] / roof['peak']
    roof['kernel'] = dominant
    roof['traffic'] = TRAFFIC_BYTES_PER_LAUNCH.get(dominant)
    roof['peak_source'] = f'{peak_kind} ({"sustained" if roof["bound"] == "tensor" else "copy"})'

    if rank != 0:
        if world > 1:
            dist.destroy_process_group()
        return

    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        v, threads, sample = cpu_sample(4, args.cpu_seconds)
        cpu = {'value': v, 'unit': 'member-samples/s', 'cores': threads, 'kind': 'port',
               'sample': sample + ' (numpy restatement of the reference layer, fp32)'}

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
        'clocks': clocks.summary(),
    }
    print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


# DRAM bytes (read + write) per full-size launch, from the ncu capture of the layer kernels
# (32-member case scaled by 256/32).
TRAFFIC_BYTES_PER_LAUNCH: dict[str, float | None] = {
    'fwd': (25.796096e6 + 212.714752e6) * 8,
    'act': (293.625344e6 + 94.327552e6) * 8,
    'dgrad': (173.594624e6 + 100.386560e6) * 8,
    'wgrad': (180.835072e6 + 42.455808e6) * 8,
}


def run_optimizer(args) -> None:
    """Grouped optimizer step: `members` x 3 weight matrices with rows and cols ~ U{64..1024
    step 16} (entries N(0, 0.02^2), gradients N(0, 1e-3^2)), one Muon group per matrix with
    5 Newton-Schulz iterations and the update scale sqrt(max(1, out/in)), plus one grouped
    AdamW launch over the matrices' bias vectors; per-member lr log-U[1e-4, 1e-2], weight
    decay log-U[1e-6, 1e-2], beta2 U[0.95, 0.999]."""
    import torch

    from tabpack_b200 import ops

    dev = torch.device('cuda', 0)
    torch.cuda.set_device(dev)
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
    adamw_ms = []

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

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    aev = [[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(args.steps)]
    with ClockSampler(0) as clocks:
        e0.record()
        for i in range(args.steps):
            step(args.warmup + i, aev[i])
        e1.record()
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    adamw_ms = statistics.mean(a.elapsed_time(b) for a, b in aev)
    peaks, kind = load_peaks()
    ach = flops / (ms / 1e3) / 1e12
    print(json.dumps({
        'metric': 'grouped Muon optimizer step (3 ragged matrices per member)', 'value': 3 * P / (ms / 1e3),
        'unit': 'matrices/s', 'ms_per_step': ms, 'steps': args.steps, 'warmup': args.warmup,
        'config': {'workload': f'{P} members x 3 matrices, rows/cols U{{64..1024 step 16}}, 5 Newton-Schulz '
                               'iterations; AdamW on the 3 bias vectors',
                   'ns_tflop_per_step': flops / 1e12, 'elements': elems,
                   'adamw': {'ms': adamw_ms, 'elements': adamw_elems,
                             'gbs': 28.0 * adamw_elems / (adamw_ms / 1e3) / 1e9,
                             'hbm_frac': 28.0 * adamw_elems / (adamw_ms / 1e3) / 1e9 / peaks['hbm_gbs']}},
        'roofline': {'bound': 'tensor', 'achieved': ach, 'peak': peaks['bf16_tflops_sustained'], 'unit': 'TFLOP/s',
                     'frac': ach / peaks['bf16_tflops_sustained'], 'peak_source': f'{kind} (sustained)',
                     'note': 'whole step (elementwise + Newton-Schulz) time against Newton-Schulz FLOPs'},
        'clocks': clocks.summary()}), flush=True)


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


def run_train(args) -> None:
    """Training steps of the full-training configuration: binary classification over
    1 000 000 synthetic rows (100 numerical features N(0, 1), 10 % of rows heavy-tailed
    Student-t(3); 10 categorical features with cardinalities log-U[2, 1000]; labels
    Bernoulli(sigmoid(random teacher MLP))); `members` members per GPU with depth U{1..4},
    width U{128..1024 step 8}, dropout U[0, 0.5], Muon + AdamW, batch 1024, bf16 autocast.
    One step = batch gather, one-hot encoding, forward, loss, backward and optimizer step of
    every member; value = member-samples/s (members x 1024 / step time)."""
    import torch

    from tabpack_b200.training import PackTrainer

    dev = torch.device('cuda', 0)
    torch.cuda.set_device(dev)
    rng = np.random.default_rng(21)
    N, n_num, batch = 1_000_000, 100, 1024
    cards = [int(c) for c in np.exp(rng.uniform(np.log(2), np.log(1000), 10)).round()]
    g = torch.Generator(device=dev).manual_seed(21)
    x = torch.randn(N, n_num, device=dev, generator=g)
    heavy = torch.rand(N, device=dev, generator=g) < 0.1
    t3 = torch.distributions.StudentT(3.0).sample((int(heavy.sum()), n_num)).to(dev)
    x[heavy] = t3
    xc = torch.stack([torch.randint(0, c, (N,), device=dev, generator=g) for c in cards], 1)
    w1 = torch.randn(n_num, 64, device=dev, generator=g) / n_num ** 0.5
    y = (torch.rand(N, device=dev, generator=g) < torch.sigmoid(torch.relu(x @ w1).sum(1) / 8 - 1)).to(torch.int64)
    data = {'x_num': x, 'x_cat': xc, 'y': y}
    P = args.members
    per = [dict(n_blocks=int(rng.integers(1, 5)), d_block=int(rng.integers(16, 129)) * 8,
                dropout=float(rng.uniform(0, 0.5))) for _ in range(P)]
    model = dict(n_numerical_features=n_num, categorical_cardinalities=cards, d_out=1, max_d_block=1024,
                 max_n_blocks=4)
    if args.embeddings == 'cosine':
        # the reference's default model: cosine numerical embeddings of per-member size
        from tabpack_b200.nn import CosineEmbeddingsPack

        model['numerical_embeddings'] = {'type': CosineEmbeddingsPack, 'max_d_embedding': 32}
        for pm in per:
            pm['numerical_embeddings'] = {'d_embedding': int(rng.integers(8, 33)),
                                          'init_scale': float(np.exp(rng.uniform(np.log(0.01), np.log(1.0))))}
    trainer = PackTrainer(n_members=P, model=model, per_member_model=per,
                          optimizer=dict(type='muon', adamw_lr=1e-3, weight_decay=1e-5, muon_lr=2e-2),
                          loss='bce', seed=0, device=dev, autocast_bf16=True, member_range=(0, P))
    steps = args.steps
    # backward on the calling thread (kernels are asynchronous either way), so that the NVTX
    # range below also holds the backward launches
    torch.autograd.set_multithreading_enabled(False)
    trainer.fit_epoch({k: v[: batch * args.warmup] for k, v in data.items()}, batch_size=batch, epoch=0)
    torch.cuda.synchronize()
    sub = {k: v[: batch * steps] for k, v in data.items()}
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(0) as clocks:
        torch.cuda.nvtx.range_push('timed')  # lets a profiler keep only the timed steps
        e0.record()
        loss = trainer.fit_epoch(sub, batch_size=batch, epoch=1)
        e1.record()
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    print(json.dumps({
        'metric': 'member-samples/sec train (full TabPack training step)', 'value': P * batch / (ms / 1e3),
        'unit': 'member-samples/s', 'n_gpus': 1, 'steps': steps, 'warmup': args.warmup, 'ms_per_step': ms,
        'higher_is_better': True, 'dtype': 'bf16', 'data': 'synthetic',
        'config': {'workload': f'{P} members, depth U{{1..4}}, width U{{128..1024}}, 100 numerical + 10 categorical '
                               f'(sum of cardinalities {sum(cards)}), batch 1024, Muon + AdamW, bf16'
                               + (', cosine numerical embeddings d U{8..32}' if args.embeddings == 'cosine' else ''),
                   'mean_train_loss': float(loss.mean())},
        'clocks': clocks.summary()}), flush=True)


def run_inference(args) -> None:
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

    world = int(os.environ.get('WORLD_SIZE', '1'))
    rank = int(os.environ.get('RANK', '0'))
    local = int(os.environ.get('LOCAL_RANK', '0'))
    torch.cuda.set_device(local)
    dev = torch.device('cuda', local)
    if world > 1:
        dist.init_process_group('nccl', device_id=dev, timeout=datetime.timedelta(seconds=120))
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
    if rank == 0:
        print(json.dumps({
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
            'clocks': clocks.summary()}), flush=True)
    if world > 1:
        dist.destroy_process_group()


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
    ap.add_argument('--steps', type=int, default=300)
    ap.add_argument('--warmup', type=int, default=10)
    ap.add_argument('--impl', choices=['b200', 'reference'], default='b200')
    ap.add_argument('--cpu-seconds', type=float, default=10.0)
    ap.add_argument('--no-cpu-baseline', action='store_true')
    ap.add_argument('--members', type=int, default=None,
                    help='members per GPU (default 256 for the layer workload, 1024 for the optimizer)')
    ap.add_argument('--workload', choices=['layer', 'optimizer', 'metrics', 'train', 'inference', 'onehot'],
                    default='layer',
                    help='layer: the packed-block fwd+bwd benchmark (default); optimizer: grouped Muon step; '
                         'metrics: validation metrics, ROC AUC and greedy selection')
    ap.add_argument('--embeddings', choices=['none', 'cosine'], default='none',
                    help='train workload: numerical features raw or through cosine embeddings')
    args = ap.parse_args()
    if args.members is None:
        args.members = {'optimizer': 1024, 'metrics': 512, 'train': 512, 'inference': 1024,
                        'onehot': 512}.get(args.workload, MEMBERS)
    MEMBERS = args.members
    if args.workload == 'optimizer':
        run_optimizer(args)
        return
    if args.workload == 'metrics':
        run_metrics(args)
        return
    if args.workload == 'train':
        run_train(args)
        return
    if args.workload == 'inference':
        run_inference(args)
        return
    if args.workload == 'onehot':
        run_onehot(args)
        return
    if args.impl == 'reference':
        run_reference(args)
    else:
        run_b200(args)


if __name__ == '__main__':
    main()
