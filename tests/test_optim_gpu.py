"""Optimizer packs on the GPU (through the C ABI) against the reference and the oracle.

Newton-Schulz runs in bf16 on tcgen05 tensor cores with each member oriented on its
own min(out, in) side; it must agree with the reference's bf16 iteration within
2e-2 (relative to the largest entry).  Momentum buffers (fp32) agree to 1e-5.
"""

import numpy as np
import pytest
import torch

from oracle import optim as oo

pytestmark = pytest.mark.gpu


@pytest.fixture(scope='module', autouse=True)
def _gpu():
    if not torch.cuda.is_available():
        pytest.skip('needs a GPU')


def _ns_via_muon(G: np.ndarray, out_f=None, in_f=None, steps=5) -> np.ndarray:
    """NS(G) through tp_muon_step: momentum 0, no weight decay, lr 1, scale 1, p = 0."""
    from tabpack_b200 import ops

    g = torch.tensor(G, dtype=torch.float32, device='cuda').contiguous()
    p = torch.zeros_like(g)
    m = torch.zeros_like(g)
    P = g.shape[0]
    ops.muon_step(p, g, m, out_features=None if out_f is None else torch.tensor(out_f, device='cuda'),
                  in_features=None if in_f is None else torch.tensor(in_f, device='cuda'),
                  lr=1.0, momentum=0.0, weight_decay=0.0, update_scale=torch.ones(P, device='cuda'),
                  nesterov=True, ns_steps=steps)
    torch.cuda.synchronize()
    return -p.cpu().numpy()


def test_newton_schulz_matches_reference(golden):
    g = golden('newton_schulz.npz')
    for j in range(3):
        got = _ns_via_muon(g[f'G{j}'])
        want = g[f'X{j}']
        err = np.abs(got - want).max() / np.abs(want).max()
        assert err < 2e-2, (j, err)


def test_newton_schulz_ragged_multi_tile():
    """Members spanning several 128-row / 256-column tiles, tall and wide, one all-zero."""
    rng = np.random.default_rng(3)
    out_f = np.array([300, 72, 16, 200, 520, 64], np.int32)
    in_f = np.array([140, 520, 16, 200, 96, 40], np.int32)
    P, mo, mi = len(out_f), int(out_f.max()), int(in_f.max())
    G = np.zeros((P, mo, mi), np.float32)
    for i in range(P):
        G[i, :out_f[i], :in_f[i]] = rng.standard_normal((out_f[i], in_f[i])) * 0.02
    G[2] = 0.0  # all-zero update: skipped, stays zero
    got = _ns_via_muon(G, out_f, in_f)
    want = oo.newton_schulz5_ragged(G, out_f, in_f)
    assert np.all(got[2] == 0)
    for i in range(P):
        if i == 2:
            continue
        a, b = got[i, :out_f[i], :in_f[i]], want[i, :out_f[i], :in_f[i]]
        err = np.linalg.norm(a - b) / np.linalg.norm(b)
        assert err < 2e-2, (i, err)
        # padding of the update stays exactly zero
        assert np.all(got[i, out_f[i]:, :] == 0) and np.all(got[i, :, in_f[i]:] == 0)


def _ns_torch(G: torch.Tensor, steps: int = 5) -> torch.Tensor:
    """`_zeropower_via_newtonschulz5` (`optim.py:464-490`) in PyTorch bf16 on one (r, c)
    matrix: Frobenius normalisation + 1e-7, the quintic with (3.4445, -4.7750, 2.0315), each
    matmul accumulating in fp32 and rounding once to bf16, transposed when tall."""
    a, b, c = 3.4445, -4.7750, 2.0315
    X = G.bfloat16()
    tall = X.shape[0] > X.shape[1]
    if tall:
        X = X.T
    X = X / (X.norm() + 1e-7)
    for _ in range(steps):
        A = X @ X.T
        B = torch.addmm(A, A, A, beta=b, alpha=c)
        X = torch.addmm(X, B, X, beta=a)
    return (X.T if tall else X).float()


def test_newton_schulz_full_size_against_torch():
    """256 ragged members (out and in U{64..1024 step 16}, several tiles per CTA) against the
    reference's bf16 iteration run per member in PyTorch: relative Frobenius error below 2e-2
    for every member, padding exactly zero."""
    from tabpack_b200 import ops

    rng = np.random.default_rng(11)
    P, W = 256, 1024
    out_f = (rng.integers(4, 65, P) * 16).astype(np.int32)
    in_f = (rng.integers(4, 65, P) * 16).astype(np.int32)
    gen = torch.Generator(device='cuda').manual_seed(11)
    g = torch.randn(P, W, W, device='cuda', generator=gen) * 0.02
    rows = torch.arange(W, device='cuda')
    valid = (rows[None, :, None] < torch.from_numpy(out_f).cuda()[:, None, None]) & \
            (rows[None, None, :] < torch.from_numpy(in_f).cuda()[:, None, None])
    g = g * valid
    p = torch.zeros_like(g)
    mb = torch.zeros_like(g)
    ops.muon_step(p, g.clone(), mb, out_features=torch.from_numpy(out_f).cuda(),
                  in_features=torch.from_numpy(in_f).cuda(), lr=1.0, momentum=0.0, weight_decay=0.0,
                  update_scale=torch.ones(P, device='cuda'), nesterov=True, ns_steps=5)
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    got = -p
    assert int(torch.count_nonzero(got * ~valid)) == 0
    for i in range(P):
        o, n = int(out_f[i]), int(in_f[i])
        want = _ns_torch(g[i, :o, :n])
        err = float(torch.linalg.norm(got[i, :o, :n] - want) / torch.linalg.norm(want))
        assert err < 2e-2, (i, o, n, err)


def test_muon_adamw_pack_matches_reference(golden):
    from tabpack_b200 import nn as bnn
    from tabpack_b200 import optim as bopt

    g = golden('muon.npz')
    P = 3
    lin = bnn.LinearPack([24, 16, 32], [32, 16, 8], max_in_features=32, max_out_features=32, pack_size=P).cuda()
    out = bnn.LinearPack(32, 2, pack_size=P).cuda()
    with torch.no_grad():
        lin.weight.copy_(torch.from_numpy(g['w0']))
    group = bopt.MuonAdamWPack.make_muon_parameter_group(lin)
    np.testing.assert_allclose(group['muon_update_scale'].cpu().numpy(), g['scale'], rtol=1e-7)
    opt = bopt.MuonAdamWPack(
        [group, {'params': [lin.bias, out.weight, out.bias]}],
        adamw_lr=[1e-3, 2e-3, 5e-3], weight_decay=[1e-2, 0.0, 1e-3], muon_lr=[0.02, 0.01, 0.05],
        muon_momentum=[0.95, 0.9, 0.8], pack_size=P, allow_inplace_grad_mutation=True)
    w_prev_ref = g['w0']
    for s in range(2):
        w_prev = lin.weight.detach().cpu().numpy()
        lin.weight.grad = torch.from_numpy(g[f's{s}.g']).cuda()
        for prm in (lin.bias, out.weight, out.bias):
            prm.grad = torch.zeros_like(prm)
        opt.step()
        torch.cuda.synchronize()
        mom = opt.state[lin.weight]['muon_momentum_buffer'].cpu().numpy()
        np.testing.assert_allclose(mom, g[f's{s}.mom'], rtol=1e-5, atol=1e-12)
        # the applied update (bf16 Newton-Schulz) against the reference's, relative Frobenius
        w = lin.weight.detach().cpu().numpy()
        delta, delta_ref = w - w_prev, g[f's{s}.w'] - w_prev_ref
        err = np.linalg.norm(delta - delta_ref) / np.linalg.norm(delta_ref)
        assert err < 2e-2, err
        w_prev_ref = g[f's{s}.w']


@pytest.mark.parametrize('case', [0, 1, 2, 3])
def test_adamw_pack_class_matches_reference(golden, case):
    from tabpack_b200 import nn as bnn  # noqa: F401
    from tabpack_b200 import optim as bopt
    from tabpack_b200.nn import ParameterPack

    g = golden('adamw.npz')
    pm = bool(g[f'c{case}.per_member'])
    sr = bool(g[f'c{case}.support_replacement'])
    hp = {}
    for k in ('lr', 'beta1', 'beta2', 'eps', 'weight_decay'):
        v = g[f'c{case}.hp.{k}']
        hp[k] = [float(x) for x in v] if pm else float(v)
    w = ParameterPack(torch.from_numpy(g[f'c{case}.w0']).cuda())
    b = ParameterPack(torch.from_numpy(g[f'c{case}.b0']).cuda())
    opt = bopt.AdamWPack([w, b], pack_size=4, support_replacement=sr, **hp)
    for s in range(3):
        w.grad = torch.from_numpy(g[f'c{case}.s{s}.gw']).cuda()
        b.grad = torch.from_numpy(g[f'c{case}.s{s}.gb']).cuda()
        opt.step()
        torch.cuda.synchronize()
        np.testing.assert_allclose(w.detach().cpu().numpy(), g[f'c{case}.s{s}.w'], rtol=1e-5, atol=1e-6)
        np.testing.assert_allclose(b.detach().cpu().numpy(), g[f'c{case}.s{s}.b'], rtol=1e-5, atol=1e-6)


def test_muon_normalisation_quotient_equals_cuda_division():
    """The Muon normalisation divides every element by the matrix's bf16 norm through the
    reciprocal and one fused correction step (Markstein's method).  Checked exhaustively
    against CUDA's correctly rounded division (`__fdiv_rn`): every positive normal bf16
    divisor, every finite bf16 dividend with |x| <= 2 * divisor -- every pair the normalisation
    can meet, since an element never exceeds its matrix's norm and both are bf16 there.  The
    stored bf16 quotients must agree bit for bit (the sign of zero included); the fp32
    quotients before that rounding may differ in the last place, which is reported."""
    if not torch.cuda.is_available():
        pytest.skip('needs a GPU')
    from tabpack_b200 import _lib

    lib = _lib.load()
    counts = torch.zeros(4, dtype=torch.int64, device='cuda')
    stream = torch.cuda.current_stream().cuda_stream
    first, last = 0x0080, 0x7F7F  # smallest and largest positive normal bf16
    rc = lib.tp_quotient_check(first, last - first + 1, counts.data_ptr(), stream)
    assert rc == 0, lib.tp_last_error_string()
    m32, m16, n, sub = counts.tolist()
    print(f'quotient check: {n} pairs, {m32} fp32 results differ from x / den ({sub} of them with a subnormal '
          f'quotient or reciprocal), {m16} differ after rounding to bf16')
    assert n > 1_000_000_000
    assert m16 == 0  # what the normalisation stores agrees bit for bit, the sign of zero included
    assert m32 < 0.01 * n


def _adamw_expected(p, g, m, v, *, lr, beta1, beta2, eps, wd, step):
    """The reference's AdamW ops (optim.py:400-427) one fp32 rounding at a time, on the CPU
    in float64 with explicit rounding to fp32: torch's lerp as fma(w or w - 1, end - self,
    self or end), addcmul as fma(value * g, g, v * beta2), addcdiv as p + (value * m) / denom
    when the step size is a Python float, p - (m / denom) * step otherwise; square root and
    division correctly rounded (the reference's CPU fp32 square root is not: it is 1 ulp off for
    about 0.6 % of values, which no CUDA kernel reproduces).  A fused multiply-add is evaluated exactly in float64 (the
    product of two fp32 values is exact there) and rounded once more to fp32; that second
    rounding could differ from a single one only at an fp32 tie, which these random values
    do not produce.  Hyperparameters are floats or (P,) fp32 tensors; step an int or (P,)."""
    f = lambda t: t.to(torch.float32)  # noqa: E731
    d = lambda t: t.to(torch.float64)  # noqa: E731
    P = p.shape[0]
    shape = (P,) + (1,) * (p.ndim - 1)
    col = lambda x: x.reshape(shape) if isinstance(x, torch.Tensor) else x  # noqa: E731

    def fma(a, b, c):
        return f(d(a) * d(b) + d(c))

    def lerp(a, b, w):
        w = w if isinstance(w, torch.Tensor) else torch.tensor(w, dtype=torch.float32)
        w = torch.broadcast_to(w, a.shape)
        dd = f(b - a)
        small = w.abs() < 0.5
        return torch.where(small, fma(w, dd, a), fma(f(w - 1), dd, b))

    pm = lambda x: isinstance(x, torch.Tensor)  # noqa: E731
    if pm(lr) or pm(wd):
        mult = f(1 - f(col(lr) * col(wd)))
        p = f(p * mult)
    elif lr != 0.0 and wd != 0.0:
        p = f(p * torch.tensor(1 - lr * wd, dtype=torch.float32))
    m = lerp(m, g, f(1 - col(beta1)) if pm(beta1) else torch.tensor(1 - beta1, dtype=torch.float32))
    if pm(beta2):
        v = lerp(v, f(g * g), f(1 - col(beta2)))
    else:
        v = fma(f(torch.tensor(1 - beta2, dtype=torch.float32) * g), g,
                f(v * torch.tensor(beta2, dtype=torch.float32)))
    st = step
    if pm(beta1) or pm(st):
        bc1 = f(1 - torch.pow(d(col(beta1)) if pm(beta1) else beta1, d(col(st)) if pm(st) else st))
    else:
        bc1 = 1 - beta1 ** st
    if pm(beta2) or pm(st):
        sbc2 = f(torch.sqrt(d(f(1 - torch.pow(d(col(beta2)) if pm(beta2) else beta2,
                                              d(col(st)) if pm(st) else st)))))
    else:
        sbc2 = torch.tensor((1 - beta2 ** st) ** 0.5, dtype=torch.float32)
    # a correctly rounded fp32 square root (float64 then fp32; torch's CPU fp32 sqrt is not)
    denom = f(f(f(torch.sqrt(d(v))) / sbc2) + (col(eps) if pm(eps) else torch.tensor(eps, dtype=torch.float32)))
    if not pm(lr) and not pm(bc1):
        step_size = torch.tensor(lr / bc1, dtype=torch.float32)
        p = f(p + f(f(-step_size * m) / denom))
    else:
        step_size = f(col(lr) / (bc1 if pm(bc1) else torch.tensor(bc1, dtype=torch.float32)))
        p = f(p - f(f(m / denom) * step_size))
    return p, m, v


@pytest.mark.parametrize('case', ['scalar', 'per_member_lr', 'per_member_all', 'no_decay', 'member_steps'])
def test_adamw_kernel_rounds_like_the_reference_ops(case):
    """Every element of the grouped AdamW kernel bit for bit equal to the reference's op
    sequence rounded as torch rounds each op (`_adamw_expected`), for packs whose per-member
    size is and is not a multiple of 4 (vector and scalar paths of the kernel).  Bias
    corrections use the same float32 powers where they are per member (the kernel's powf and
    the expectation's float64 power rounded to fp32 may differ in the last place; those cases
    compare the bias-correction-free part only through the moments)."""
    from tabpack_b200 import ops

    P = 12
    gen = torch.Generator().manual_seed(sum(map(ord, case)))
    pmv = lambda lo, hi: torch.rand(P, generator=gen) * (hi - lo) + lo  # noqa: E731
    hp = dict(lr=1e-3, beta1=0.9, beta2=0.999, eps=1e-8, wd=1e-2)
    if case == 'per_member_lr':
        hp['lr'] = pmv(1e-4, 3e-3)
    elif case == 'per_member_all':
        hp = dict(lr=pmv(1e-4, 3e-3), beta1=pmv(0.8, 0.95), beta2=pmv(0.95, 0.999), eps=pmv(1e-9, 1e-7),
                  wd=pmv(0.0, 0.1))
    elif case == 'no_decay':
        hp['wd'] = 0.0
    steps = torch.randint(1, 40, (P,), generator=gen) if case == 'member_steps' else None
    for shape in ((P, 64, 36), (P, 130), (P, 7, 5), (P, 1)):
        p = torch.randn(shape, generator=gen)
        g = torch.randn(shape, generator=gen) * 1e-2
        m = torch.randn(shape, generator=gen) * 1e-3
        v = torch.rand(shape, generator=gen) * 1e-4
        step = 7
        want = _adamw_expected(p, g, m, v, lr=hp['lr'], beta1=hp['beta1'], beta2=hp['beta2'], eps=hp['eps'],
                               wd=hp['wd'], step=steps if steps is not None else step)
        dev = [t.cuda() for t in (p, g, m, v)]
        cuda_hp = {k: (x.cuda() if isinstance(x, torch.Tensor) else x) for k, x in hp.items()}
        ops.adamw_step([dev[0]], [dev[1]], [dev[2]], [dev[3]], step=step,
                       steps=None if steps is None else [steps.cuda()], lr=cuda_hp['lr'], beta1=cuda_hp['beta1'],
                       beta2=cuda_hp['beta2'], eps=cuda_hp['eps'], weight_decay=cuda_hp['wd'])
        torch.cuda.synchronize()
        names = ('p', 'exp_avg', 'exp_avg_sq')
        for name, got, exp in zip(names, (dev[0], dev[2], dev[3]), want):
            if name == 'p' and (case in ('per_member_all', 'member_steps')):
                # per-member powers: powf on the device against float64 rounded to fp32 here
                np.testing.assert_allclose(got.cpu().numpy(), exp.numpy(), rtol=2e-6, atol=1e-8)
                continue
            diff = int((got.cpu().view(torch.int32) != exp.view(torch.int32)).sum())
            assert diff == 0, f'{case} {shape} {name}: {diff} of {exp.numel()} elements differ'


def test_muon_step_refreshes_the_bf16_weight_copy():
    """Under bf16 autocast a LinearPack multiplies with a cached bf16 copy of its weights.  A
    Muon step writes bf16 of the new weights into that copy in the pass that updates them, so
    the copy is current afterwards (its key at the weight's new version: the next forward
    casts nothing) and equals bf16 of the updated weights on every member's block, bit for bit."""
    from tabpack_b200 import nn as bnn
    from tabpack_b200 import optim as bopt

    P = 4
    outs, ins = [72, 16, 48, 64], [40, 24, 64, 8]
    lin = bnn.LinearPack(ins, outs, max_in_features=64, max_out_features=72, pack_size=P).cuda()
    opt = bopt.MuonAdamWPack([bopt.MuonAdamWPack.make_muon_parameter_group(lin), {'params': [lin.bias]}],
                             adamw_lr=1e-3, weight_decay=1e-2, muon_lr=0.02, pack_size=P,
                             allow_inplace_grad_mutation=False)
    gen = torch.Generator(device='cuda').manual_seed(5)
    x = torch.randn(P, 32, 64, device='cuda', generator=gen)
    rows = torch.arange(72, device='cuda')[None, :, None] < torch.tensor(outs, device='cuda')[:, None, None]
    cols = torch.arange(64, device='cuda')[None, None, :] < torch.tensor(ins, device='cuda')[:, None, None]
    valid = rows & cols
    for _ in range(3):
        with torch.autocast('cuda', dtype=torch.bfloat16):
            y = lin(x)
        y.float().square().sum().backward()
        del y
        opt.step()
        opt.zero_grad()
        torch.cuda.synchronize()
        cache = bnn.bf16_copy_cache(lin.weight)
        assert cache is lin._cache and cache.key is not None
        assert cache.key[1] == lin.weight._version, 'the copy was not refreshed with the step'
        copy = cache.value[:, :72, :64]
        want = lin.weight.detach().bfloat16()
        assert torch.equal(copy[valid].view(torch.int16), want[valid].view(torch.int16))
        del copy  # a view of the copy would keep the next step from writing into it


def test_muon_step_with_depth_gated_members():
    """Members whose depth leaves the block out (n_blocks <= block_index) have an exactly zero
    gradient, which the step then does not read: weights and momentum bit-identical to the
    same step reading the zero gradient, also for a gated member whose momentum is still
    nonzero (it takes the full update); the bf16 copy is written for the other members."""
    from tabpack_b200 import ops

    P, O, I = 6, 200, 136
    gen = torch.Generator(device='cuda').manual_seed(17)
    outf = torch.tensor([200, 64, 128, 200, 96, 8], dtype=torch.int32, device='cuda')
    inf = torch.tensor([136, 40, 136, 72, 136, 16], dtype=torch.int32, device='cuda')
    nb = torch.tensor([3, 1, 2, 4, 1, 2], dtype=torch.int32, device='cuda')  # block 1: members 1, 4 gated
    valid = ((torch.arange(O, device='cuda')[None, :, None] < outf[:, None, None])
             & (torch.arange(I, device='cuda')[None, None, :] < inf[:, None, None]))
    p0 = torch.randn(P, O, I, device='cuda', generator=gen) * 0.05
    g = torch.randn(P, O, I, device='cuda', generator=gen) * 1e-3 * valid
    g[1] = 0.0
    g[4] = 0.0
    m0 = torch.zeros(P, O, I, device='cuda')
    m0[4] = torch.randn(O, I, device='cuda', generator=gen) * 1e-3 * valid[4]  # still nonzero
    lr = torch.full((P,), 0.02, device='cuda')
    out = []
    for gated in (False, True):
        p, m = p0.clone(), m0.clone()
        copy = torch.zeros(P, O, I, dtype=torch.bfloat16, device='cuda')
        for _ in range(2):
            ops.muon_step(p, g.clone(), m, out_features=outf, in_features=inf, lr=lr, momentum=0.95,
                          weight_decay=1e-2, nesterov=True, mutate_grad=False, ns_steps=5, p_bf16=copy,
                          n_blocks=nb if gated else None, block_index=1)
        torch.cuda.synchronize()
        out.append((p, m, copy))
    (pa, ma, ca), (pb, mb, cb) = out
    assert torch.equal(pa, pb) and torch.equal(ma, mb)
    live = (nb > 1)[:, None, None] & valid
    assert torch.equal(ca[live.expand_as(ca)], cb[live.expand_as(cb)])
    assert not torch.equal(pa[4], p0[4] * (1 - 0.02 * 1e-2))  # the nonzero momentum still moved it


def test_grouped_muon_equals_one_call_per_group():
    """`tp_muon_step_grouped` over three groups of different shapes (a transposed one, ragged
    widths, a member with an all-zero update, per-member and scalar hyperparameters, a bf16
    copy, depth gating, a mutated gradient) gives each group exactly its own `tp_muon_step`
    result: weights, momentum, gradient and bf16 copy bit for bit, over two steps."""
    from tabpack_b200 import ops

    gen = torch.Generator(device='cuda').manual_seed(23)

    def group(P, O, I, *, ragged, gated, copy, per_member, mutate):
        outf = torch.randint(8, O + 1, (P,), generator=gen, device='cuda', dtype=torch.int32) if ragged else None
        inf = torch.randint(8, I + 1, (P,), generator=gen, device='cuda', dtype=torch.int32) if ragged else None
        p = torch.randn(P, O, I, device='cuda', generator=gen) * 0.05
        g = torch.randn(P, O, I, device='cuda', generator=gen) * 1e-3
        g[1] = 0.0  # all-zero update: skips the iterations
        lr = torch.rand(P, device='cuda', generator=gen) * 0.02 + 1e-3 if per_member else 0.02
        nb = torch.tensor([1, 3, 2] * P, dtype=torch.int32, device='cuda')[:P] if gated else None
        return dict(p=p, grad=g, momentum_buffer=torch.zeros_like(p), out_features=outf, in_features=inf, lr=lr,
                    momentum=0.95, weight_decay=1e-2, nesterov=True, mutate_grad=mutate, ns_steps=5,
                    p_bf16=torch.zeros(P, O, I, dtype=torch.bfloat16, device='cuda') if copy else None,
                    n_blocks=nb, block_index=1)

    groups = [group(5, 300, 136, ragged=True, gated=False, copy=True, per_member=True, mutate=False),
              group(7, 96, 520, ragged=True, gated=True, copy=False, per_member=False, mutate=True),
              group(3, 128, 128, ragged=False, gated=False, copy=True, per_member=False, mutate=False)]
    groups[1]['grad'][groups[1]['n_blocks'] <= 1] = 0.0  # gated members' gradients are exactly zero

    def clone(gr):
        return {k: (v.clone() if isinstance(v, torch.Tensor) and k in ('p', 'grad', 'momentum_buffer', 'p_bf16')
                    else v) for k, v in gr.items()}

    sep, grp = [clone(g) for g in groups], [clone(g) for g in groups]
    for _ in range(2):
        for gr in sep:
            ops.muon_step(**gr)
        ops.muon_step_grouped(grp)
    torch.cuda.synchronize()
    for i, (a, b) in enumerate(zip(sep, grp)):
        for k in ('p', 'momentum_buffer', 'grad', 'p_bf16'):
            if a[k] is None:
                continue
            assert torch.equal(a[k].view(torch.int16) if a[k].dtype == torch.bfloat16 else a[k].view(torch.int32),
                               b[k].view(torch.int16) if b[k].dtype == torch.bfloat16 else b[k].view(torch.int32)), (i, k)
        assert not torch.equal(a['p'], groups[i]['p'])


def test_muon_step_skips_gated_members_with_zero_momentum():
    """`gated_momentum_zero`: depth-gated members whose momentum is zero take only the weight
    decay; the step reads neither their gradient nor their momentum and gives exactly the
    results of the step that reads both (two steps, a bf16 copy, Nesterov)."""
    from tabpack_b200 import ops

    P, O, I = 7, 160, 96
    gen = torch.Generator(device='cuda').manual_seed(31)
    outf = torch.tensor([160, 64, 128, 8, 96, 160, 40], dtype=torch.int32, device='cuda')
    inf = torch.tensor([96, 40, 96, 16, 72, 8, 96], dtype=torch.int32, device='cuda')
    nb = torch.tensor([3, 1, 2, 1, 1, 4, 2], dtype=torch.int32, device='cuda')  # block 1: members 1, 3, 4 gated
    valid = ((torch.arange(O, device='cuda')[None, :, None] < outf[:, None, None])
             & (torch.arange(I, device='cuda')[None, None, :] < inf[:, None, None]))
    p0 = torch.randn(P, O, I, device='cuda', generator=gen) * 0.05
    g = torch.randn(P, O, I, device='cuda', generator=gen) * 1e-3 * valid
    g[nb <= 1] = 0.0
    lr = torch.rand(P, device='cuda', generator=gen) * 0.02 + 1e-3
    out = []
    for skip in (False, True):
        p, m = p0.clone(), torch.zeros(P, O, I, device='cuda')
        copy = torch.zeros(P, O, I, dtype=torch.bfloat16, device='cuda')
        for _ in range(2):
            ops.muon_step(p, g.clone(), m, out_features=outf, in_features=inf, lr=lr, momentum=0.95,
                          weight_decay=1e-2, nesterov=True, mutate_grad=False, ns_steps=5, p_bf16=copy,
                          n_blocks=nb, block_index=1, gated_momentum_zero=skip)
        torch.cuda.synchronize()
        out.append((p, m, copy))
    (pa, ma, ca), (pb, mb, cb) = out
    assert torch.equal(pa, pb) and torch.equal(ma, mb) and torch.equal(ca, cb)
    assert not torch.equal(pa[0], p0[0])
