"""Parity of the packed-linear CUDA kernels (called through the C ABI) with the oracle.

bf16 runs on tcgen05 tensor cores: inputs are bf16-exact, so the reference is the
oracle evaluated in float64 on the same bf16 values, and the only error left is
fp32 accumulation plus one bf16 rounding of each output (tolerance 2^-7
relative, far inside the 2e-2 bar).  fp32 runs on CUDA cores and must agree with
the oracle to 1e-5 relative (the bar is 1e-4).
"""

import math

import numpy as np
import pytest
import torch

from oracle import layers as ol
from oracle.philox import dropout_keep_mask, keep_scale

pytestmark = pytest.mark.gpu

BF16_RTOL = 2.0 ** -7


@pytest.fixture(scope='module', autouse=True)
def _lib():
    if not torch.cuda.is_available():
        pytest.skip('needs a GPU')
    from tabpack_b200 import _lib as L

    L.load()


def _bf16(a: np.ndarray) -> np.ndarray:
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).bfloat16().float().numpy().astype(np.float64)


def _dev(a, dtype):
    return torch.from_numpy(np.ascontiguousarray(a)).to(device='cuda', dtype=dtype)


def _host(t):
    return t.float().cpu().numpy().astype(np.float64)


def _close(got, want, rtol, what):
    scale = max(np.abs(want).max(), 1e-30)
    err = np.abs(got - want)
    bad = err > rtol * np.abs(want) + rtol * 0.25 * scale
    assert not bad.any(), f'{what}: {bad.sum()} / {bad.size} mismatches, max err {err.max():.3e} (scale {scale:.3e})'


def make_case(P, B, max_in, max_out, in_f=None, out_f=None, shared=False, seed=0, p_max=0.5):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((1 if shared else P, B, max_in))
    if in_f is not None and not shared:
        x = x * (np.arange(max_in)[None, None, :] < np.asarray(in_f)[:, None, None])
    fan = np.asarray(in_f if in_f is not None else [max_in] * P, np.float64)
    w = rng.uniform(-1, 1, (P, max_out, max_in)) / np.sqrt(fan)[:, None, None]
    b = rng.uniform(-1, 1, (P, max_out)) / np.sqrt(fan)[:, None]
    p = rng.uniform(0, p_max, P).astype(np.float32)
    p[0] = 0.0
    return x, w, b, p


def oracle_forward(x, w, b, out_f, p, seed, offset, member_base, B, relu=True, dropout=True, bf16=False):
    """The block forward in fp64 (the kernels round each output to bf16 once)."""
    P, max_out, _ = w.shape
    mv = None
    if dropout:
        mv = ol.dropout_mask_values(seed=seed, offset=offset, members=np.arange(P) + member_base,
                                    n_rows=B, n_cols=max_out, p=p, dtype=np.float64)
    xx = x if x.shape[0] == P else np.broadcast_to(x, (P, *x.shape[1:]))
    del bf16
    y, _ = ol.block_forward(xx, w, b, out_f, mask_values=mv, relu=relu)
    return y, mv


@pytest.mark.parametrize('P,B,cols,seed,offset,base', [(3, 37, 50, 1, 0, 0), (5, 130, 264, 2**40 + 7, 9, 1000)])
def test_dropout_mask_bit_exact(P, B, cols, seed, offset, base):
    from tabpack_b200 import ops

    p = np.array([0.0, 0.1, 0.37, 0.5, 0.99][:P], np.float32)
    got = ops.dropout_mask(seed=seed, offset=offset, member_base=base, p=_dev(p, torch.float32), rows=B, cols=cols)
    want = dropout_keep_mask(seed=seed, offset=offset, members=np.arange(P) + base, n_rows=B, n_cols=cols, p=p)
    assert np.array_equal(got.cpu().numpy().astype(bool), want)


CASES = [
    # P, B, max_in, max_out, in_f, out_f, shared
    (3, 300, 72, 520, [72, 16, 40], [520, 16, 264], False),
    (2, 128, 512, 1024, None, None, False),
    (4, 200, 64, 256, None, [256, 8, 136, 200], True),
    (2, 77, 24, 40, [24, 9], [40, 33], False),
]


@pytest.mark.parametrize('dtype', [torch.bfloat16, torch.float32])
@pytest.mark.parametrize('case', range(len(CASES)))
@pytest.mark.parametrize('dropout', [True, False])
def test_forward(dtype, case, dropout):
    from tabpack_b200 import ops

    P, B, max_in, max_out, in_f, out_f, shared = CASES[case]
    x, w, b, p = make_case(P, B, max_in, max_out, in_f, out_f, shared, seed=case)
    if dtype == torch.bfloat16:
        x, w = _bf16(x), _bf16(w)
    seed, offset, base = 1234567 + case, 3, 17
    y = ops.linear_forward(
        _dev(x[0] if shared else x, dtype), _dev(w, dtype), _dev(b, torch.float32),
        in_features=None if in_f is None else _dev(np.array(in_f), torch.int32),
        out_features=None if out_f is None else _dev(np.array(out_f), torch.int32),
        relu=True, dropout_p=_dev(p, torch.float32) if dropout else None,
        seed=seed, offset=offset, member_base=base)
    torch.cuda.synchronize()
    want, _ = oracle_forward(x, w, b.astype(np.float32).astype(np.float64), out_f, p, seed, offset, base, B,
                             dropout=dropout, bf16=dtype == torch.bfloat16)
    _close(_host(y), want, BF16_RTOL if dtype == torch.bfloat16 else 1e-5, f'y case {case}')


def test_plain_gemm_matches_torch_fp32():
    """No widths, no activation: the tcgen05 GEMM against torch's fp32 matmul."""
    from tabpack_b200 import ops

    torch.manual_seed(0)
    P, B, K, N = 3, 384, 320, 512
    x = torch.randn(P, B, K, device='cuda').bfloat16()
    w = torch.randn(P, N, K, device='cuda').bfloat16() / K ** 0.5
    y = ops.linear_forward(x, w, None)
    ref = torch.bmm(x.float(), w.float().transpose(1, 2))
    err = (y.float() - ref).abs().max().item() / ref.abs().max().item()
    assert err < 2 ** -7, err


@pytest.mark.parametrize('dtype', [torch.bfloat16, torch.float32])
@pytest.mark.parametrize('case', range(len(CASES)))
def test_backward(dtype, case):
    from tabpack_b200 import ops

    P, B, max_in, max_out, in_f, out_f, shared = CASES[case]
    x, w, b, p = make_case(P, B, max_in, max_out, in_f, out_f, shared, seed=10 + case)
    if dtype == torch.bfloat16:
        x, w = _bf16(x), _bf16(w)
    seed, offset, base = 99, 1, 0
    kw = dict(in_features=None if in_f is None else _dev(np.array(in_f), torch.int32),
              out_features=None if out_f is None else _dev(np.array(out_f), torch.int32),
              relu=True, dropout_p=_dev(p, torch.float32), seed=seed, offset=offset, member_base=base)
    xd, wd = _dev(x[0] if shared else x, dtype), _dev(w, dtype)
    y = ops.linear_forward(xd, wd, _dev(b, torch.float32), **kw)
    rng = np.random.default_rng(case)
    dy = rng.standard_normal((P, B, max_out))
    if dtype == torch.bfloat16:
        dy = _bf16(dy)
    dx, dW, db = ops.linear_backward(_dev(dy, dtype), xd, wd, y, **kw)
    torch.cuda.synchronize()
    # reference gradient w.r.t. the pre-activation, using the kernel's own y for the ReLU mask
    mv = ol.dropout_mask_values(seed=seed, offset=offset, members=np.arange(P), n_rows=B, n_cols=max_out,
                                p=p, dtype=np.float64)
    yh = _host(y)
    g = dy * mv * (yh > 0)
    if out_f is not None:
        g = g * ol.col_mask(out_f, max_out, np.float64)
    gq = _bf16(g) if dtype == torch.bfloat16 else g
    xb = np.broadcast_to(x, (P, B, max_in))
    tol = BF16_RTOL if dtype == torch.bfloat16 else 1e-5
    _close(_host(db), g.sum(1), 1e-4 if dtype == torch.bfloat16 else 1e-5, 'db')
    _close(_host(dW), np.matmul(np.swapaxes(gq, 1, 2), xb), tol, 'dW')
    dx_ref = np.matmul(gq, w)
    if in_f is not None:
        dx_ref = dx_ref * ol.col_mask(in_f, max_in, np.float64)
    _close(_host(dx), dx_ref, tol, 'dx')


def _close_dev(got, want, rtol, what):
    """`_close` on the device: |got - want| <= rtol |want| + rtol / 4 * max |want|."""
    got, want = got.float(), want.float()
    scale = want.abs().max().clamp_min(1e-30)
    err = (got - want).abs()
    n = int((err > rtol * want.abs() + rtol * 0.25 * scale).sum())
    assert n == 0, f'{what}: {n} / {err.numel()} mismatches, max err {float(err.max()):.3e} (scale {float(scale):.3e})'


@pytest.mark.parametrize('dropout', [True, False])
def test_full_size_layer_against_torch_fp32(dropout):
    """The benchmarked layer at full size: 256 members sharing a 4096 x 512 bf16 batch, output
    widths U{64..1024 step 16}, bias + ReLU + dropout p ~ U[0, 0.5] (without dropout the
    forward runs on CTA pairs).  Every member's output,
    input gradient, weight gradient and bias gradient against plain PyTorch fp32 arithmetic on
    the same bf16 values (TF32 off), with the ReLU mask taken from the kernel's own output as in
    `test_backward`; exact zeros in every member's padding; and the keep masks of sampled
    members (first, last, narrowest, widest) bit-exact against the oracle's Philox."""
    from tabpack_b200 import ops

    P, B, K, N = 256, 4096, 512, 1024
    rng = np.random.default_rng(2024)
    out_np = rng.integers(4, 65, P) * 16
    p_np = rng.uniform(0, 0.5, P).astype(np.float32)
    outf = torch.from_numpy(out_np.astype(np.int32)).cuda()
    p = torch.from_numpy(p_np).cuda()
    g = torch.Generator(device='cuda').manual_seed(2024)
    bound = 1.0 / math.sqrt(K)
    x = torch.randn(B, K, device='cuda', generator=g).bfloat16()
    w = ((torch.rand(P, N, K, device='cuda', generator=g) * 2 - 1) * bound).bfloat16()
    b = (torch.rand(P, N, device='cuda', generator=g) * 2 - 1) * bound
    seed, offset, base = 0x123456789ABC, 7, 0
    kw = dict(out_features=outf, relu=True, dropout_p=p if dropout else None, seed=seed, offset=offset,
              member_base=base)
    y = ops.linear_forward(x, w, b, **kw)
    dy = torch.randn(P, B, N, device='cuda', generator=g).bfloat16()
    dx, dW, db = ops.linear_backward(dy, x, w, y, **kw)
    if dropout:
        keep = ops.dropout_mask(seed=seed, offset=offset, member_base=base, p=p, rows=B, cols=N)
    else:
        p_np = np.zeros_like(p_np)
        keep = torch.ones(P, B, N, dtype=torch.uint8, device='cuda')
    torch.cuda.synchronize()
    assert ops.device_error() == 0

    for m in sorted({0, P - 1, int(np.argmin(out_np)), int(np.argmax(out_np))}) if dropout else []:
        want = dropout_keep_mask(seed=seed, offset=offset, members=np.array([m + base]), n_rows=B, n_cols=N,
                                 p=p_np[m:m + 1])[0]
        assert np.array_equal(keep[m].cpu().numpy().astype(bool), want), f'keep mask of member {m}'

    scale = torch.from_numpy(keep_scale(p_np)).cuda()
    col = torch.arange(N, device='cuda')
    xf = x.float()
    tf32 = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        for c in range(0, P, 32):
            s = slice(c, c + 32)
            valid = (col[None, :] < outf[s, None])[:, None, :]
            mv = keep[s].float() * scale[s, None, None] * valid
            pre = torch.matmul(xf, w[s].float().transpose(1, 2)) + b[s, None, :]
            _close_dev(y[s], torch.relu(pre) * mv, BF16_RTOL, f'y members {c}..{c + 31}')
            assert int(torch.count_nonzero(y[s] * ~valid)) == 0
            gm = dy[s].float() * mv * (y[s] > 0)
            _close_dev(db[s], gm.sum(1), 1e-4, f'db members {c}..{c + 31}')
            gq = gm.bfloat16().float()
            _close_dev(dW[s], torch.matmul(gq.transpose(1, 2), xf), BF16_RTOL, f'dW members {c}..{c + 31}')
            _close_dev(dx[s], torch.matmul(gq, w[s].float()), BF16_RTOL, f'dx members {c}..{c + 31}')
            rows_pad = (col[None, :] >= outf[s, None])
            assert int(torch.count_nonzero(dW[s] * rows_pad[:, :, None])) == 0
            assert int(torch.count_nonzero(db[s] * rows_pad)) == 0
    finally:
        torch.backends.cuda.matmul.allow_tf32 = tf32


def test_long_k_forward_with_dropout_on_cta_pairs():
    """A forward with dropout whose K loop is long (2544 padded inputs, 2538 valid, as in a
    TabPack's first layer over its one-hot columns) runs on CTA pairs: every member's output
    against plain PyTorch fp32 on the same bf16 values with the library's keep mask, that mask
    bit-exact against the oracle's Philox for sampled members, exact zeros in the padding."""
    from tabpack_b200 import ops

    P, B, K, N = 24, 1024, 2544, 1024
    rng = np.random.default_rng(77)
    out_np = rng.integers(16, 129, P) * 8
    p_np = rng.uniform(0, 0.5, P).astype(np.float32)
    outf = torch.from_numpy(out_np.astype(np.int32)).cuda()
    inf = torch.full((P,), 2538, dtype=torch.int32, device='cuda')
    p = torch.from_numpy(p_np).cuda()
    g = torch.Generator(device='cuda').manual_seed(77)
    bound = 1.0 / math.sqrt(2538)
    kin = (torch.arange(K, device='cuda') < 2538)
    x = (torch.randn(P, B, K, device='cuda', generator=g) * kin).bfloat16()
    w = ((torch.rand(P, N, K, device='cuda', generator=g) * 2 - 1) * bound * kin).bfloat16()
    b = (torch.rand(P, N, device='cuda', generator=g) * 2 - 1) * bound
    seed, offset, base = 99, 3, 5
    y = ops.linear_forward(x, w, b, in_features=inf, out_features=outf, relu=True, dropout_p=p, seed=seed,
                           offset=offset, member_base=base)
    keep = ops.dropout_mask(seed=seed, offset=offset, member_base=base, p=p, rows=B, cols=N)
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    for m in (0, P - 1, int(np.argmin(out_np))):
        want = dropout_keep_mask(seed=seed, offset=offset, members=np.array([m + base]), n_rows=B, n_cols=N,
                                 p=p_np[m:m + 1])[0]
        assert np.array_equal(keep[m].cpu().numpy().astype(bool), want), f'keep mask of member {m}'
    scale = torch.from_numpy(keep_scale(p_np)).cuda()
    col = torch.arange(N, device='cuda')
    tf32 = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        for c in range(0, P, 8):
            s = slice(c, c + 8)
            valid = (col[None, :] < outf[s, None])[:, None, :]
            mv = keep[s].float() * scale[s, None, None] * valid
            pre = torch.matmul(x[s].float(), w[s].float().transpose(1, 2)) + b[s, None, :]
            _close_dev(y[s], torch.relu(pre) * mv, BF16_RTOL, f'y members {c}..{c + 7}')
            assert int(torch.count_nonzero(y[s] * ~valid)) == 0
    finally:
        torch.backends.cuda.matmul.allow_tf32 = tf32


@pytest.mark.parametrize('dropout', [True, False])
def test_depth_gating_many_tiles_per_cta(dropout):
    """128 members x 2048 rows x 512, a third of them past their depth (COPY tiles mixed with
    MMA tiles on every CTA; without dropout the forward runs on CTA pairs): gated members pass
    x and dy through bit for bit, the others match plain PyTorch fp32 on the same bf16 values
    (TF32 off)."""
    from tabpack_b200 import ops

    P, B, W = 128, 2048, 512
    rng = np.random.default_rng(21)
    nb = rng.integers(1, 4, P).astype(np.int32)
    p_np = rng.uniform(0, 0.5, P).astype(np.float32) if dropout else np.zeros(P, np.float32)
    g = torch.Generator(device='cuda').manual_seed(21)
    x = torch.randn(P, B, W, device='cuda', generator=g).bfloat16()
    bound = 1.0 / math.sqrt(W)
    w = ((torch.rand(P, W, W, device='cuda', generator=g) * 2 - 1) * bound).bfloat16()
    b = (torch.rand(P, W, device='cuda', generator=g) * 2 - 1) * bound
    p = torch.from_numpy(p_np).cuda()
    seed, offset = 77, 3
    kw = dict(n_blocks=torch.from_numpy(nb).cuda(), block_index=1, relu=True, dropout_p=p if dropout else None,
              seed=seed, offset=offset)
    y = ops.linear_forward(x, w, b, **kw)
    dy = torch.randn(P, B, W, device='cuda', generator=g).bfloat16()
    dx, dW, db = ops.linear_backward(dy, x, w, y, **kw)
    keep = ops.dropout_mask(seed=seed, offset=offset, member_base=0, p=p, rows=B, cols=W)
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    gated = torch.from_numpy(nb <= 1).cuda()
    assert torch.equal(y[gated], x[gated]) and torch.equal(dx[gated], dy[gated])
    assert int(torch.count_nonzero(dW[gated])) == 0 and int(torch.count_nonzero(db[gated])) == 0
    act = ~gated
    scale = torch.from_numpy(keep_scale(p_np)).cuda()[act][:, None, None]
    mv = keep[act].float() * scale
    tf32 = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        xa, wa = x[act].float(), w[act].float()
        pre = torch.matmul(xa, wa.transpose(1, 2)) + b[act][:, None, :]
        _close_dev(y[act], torch.relu(pre) * mv, BF16_RTOL, 'y of active members')
        gm = dy[act].float() * mv * (y[act] > 0)
        _close_dev(db[act], gm.sum(1), 1e-4, 'db of active members')
        gq = gm.bfloat16().float()
        _close_dev(dW[act], torch.matmul(gq.transpose(1, 2), xa), BF16_RTOL, 'dW of active members')
        _close_dev(dx[act], torch.matmul(gq, wa), BF16_RTOL, 'dx of active members')
    finally:
        torch.backends.cuda.matmul.allow_tf32 = tf32


def test_depth_gating_with_widths_copies_only_valid_columns():
    """Depth-gated members with their own widths (a hidden block: in = out = width): y = x and
    dx = dy bit for bit, where x and dy hold zeros beyond the member's width as a pack's
    activations do; the copy reads only the valid column tiles and writes zeros beyond."""
    from tabpack_b200 import ops

    P, B, W = 8, 300, 768
    gen = torch.Generator(device='cuda').manual_seed(8)
    widths = torch.tensor([64, 768, 200, 512, 256, 8, 520, 384], dtype=torch.int32, device='cuda')
    nb = torch.tensor([1, 2, 1, 3, 1, 1, 2, 1], dtype=torch.int32, device='cuda')
    cols = torch.arange(W, device='cuda')[None, None, :] < widths[:, None, None]
    x = (torch.randn(P, B, W, device='cuda', generator=gen) * cols).bfloat16()
    w = (torch.randn(P, W, W, device='cuda', generator=gen) * 0.03).bfloat16()
    b = torch.randn(P, W, device='cuda', generator=gen) * 0.01
    p = torch.full((P,), 0.2, device='cuda')
    kw = dict(in_features=widths, out_features=widths, n_blocks=nb, block_index=1, relu=True, dropout_p=p,
              seed=3, offset=1)
    y = ops.linear_forward(x, w, b, **kw)
    dy = (torch.randn(P, B, W, device='cuda', generator=gen) * cols).bfloat16()
    dx, dW, db = ops.linear_backward(dy, x, w, y, **kw)
    torch.cuda.synchronize()
    gated = nb <= 1
    assert torch.equal(y[gated], x[gated])
    assert torch.equal(dx[gated], dy[gated])
    assert int(torch.count_nonzero(y * ~cols)) == 0 and int(torch.count_nonzero(dx * ~cols)) == 0


@pytest.mark.parametrize('dtype', [torch.bfloat16, torch.float32])
def test_depth_gating(dtype):
    """Members with n_blocks <= block_index pass x through (forward) and dy through (dgrad)."""
    from tabpack_b200 import ops

    P, B, W = 4, 150, 192
    x, w, b, p = make_case(P, B, W, W, seed=5)
    if dtype == torch.bfloat16:
        x, w = _bf16(x), _bf16(w)
    nb = np.array([1, 2, 3, 1], np.int32)
    kw = dict(n_blocks=_dev(nb, torch.int32), block_index=1, relu=True, dropout_p=_dev(p, torch.float32),
              seed=5, offset=2)
    xd, wd = _dev(x, dtype), _dev(w, dtype)
    y = ops.linear_forward(xd, wd, _dev(b, torch.float32), **kw)
    dy = _dev(np.random.default_rng(1).standard_normal((P, B, W)), dtype)
    dx, dW, db = ops.linear_backward(dy, xd, wd, y, **kw)
    torch.cuda.synchronize()
    want, _ = oracle_forward(x, w, b.astype(np.float32).astype(np.float64), None, p, 5, 2, 0, B,
                             bf16=dtype == torch.bfloat16)
    tol = BF16_RTOL if dtype == torch.bfloat16 else 1e-5
    for m in range(P):
        if nb[m] > 1:
            _close(_host(y[m]), want[m], tol, f'y[{m}]')
        else:
            assert torch.equal(y[m], xd[m])
            assert torch.equal(dx[m], dy[m])
            assert torch.count_nonzero(dW[m]) == 0 and torch.count_nonzero(db[m]) == 0


def test_golden_block_fp32(golden):
    """The fp32 path against the reference's own outputs and gradients."""
    from tabpack_b200 import ops

    g = golden('block_fp32.npz')
    P, B, max_in = g['x'].shape
    kw = dict(in_features=_dev(g['in_features'], torch.int32), out_features=_dev(g['out_features'], torch.int32),
              relu=True, dropout_p=_dev(g['p'], torch.float32), seed=int(g['seed']), offset=int(g['offset']))
    xd, wd = _dev(g['x'], torch.float32), _dev(g['weight'], torch.float32)
    y = ops.linear_forward(xd, wd, _dev(g['bias'], torch.float32), **kw)
    dx, dW, db = ops.linear_backward(_dev(g['dy'], torch.float32), xd, wd, y, **kw)
    torch.cuda.synchronize()
    _close(_host(y), g['y'], 1e-5, 'y')
    _close(_host(dW), g['dweight'], 1e-5, 'dW')
    _close(_host(db), g['dbias'], 1e-5, 'db')
    # the reference's dx carries products with random pad weights beyond in_features;
    # those columns are masked by the previous layer and are zero here
    m = ol.col_mask(g['in_features'], max_in, np.float64)
    _close(_host(dx), g['dx'] * m, 1e-5, 'dx')


@pytest.mark.parametrize('case', [0, 1, 2, 3])
def test_adamw_golden(golden, case):
    from tabpack_b200 import ops

    g = golden('adamw.npz')
    pm = bool(g[f'c{case}.per_member'])
    sr = bool(g[f'c{case}.support_replacement'])
    hp = {}
    for k in ('lr', 'beta1', 'beta2', 'eps', 'weight_decay'):
        v = g[f'c{case}.hp.{k}']
        hp[k] = _dev(v.astype(np.float32), torch.float32) if pm else float(v)
    w = _dev(g[f'c{case}.w0'], torch.float32)
    b = _dev(g[f'c{case}.b0'], torch.float32)
    ms = [torch.zeros_like(w), torch.zeros_like(b)]
    vs = [torch.zeros_like(w), torch.zeros_like(b)]
    steps = [torch.zeros(w.shape[0], dtype=torch.int64, device='cuda') for _ in range(2)]
    for s in range(3):
        gw, gb = _dev(g[f'c{case}.s{s}.gw'], torch.float32), _dev(g[f'c{case}.s{s}.gb'], torch.float32)
        for st in steps:
            st += 1
        ops.adamw_step([w, b], [gw, gb], ms, vs, steps=steps if sr else None, step=s + 1, **hp)
        torch.cuda.synchronize()
        np.testing.assert_allclose(w.cpu().numpy(), g[f'c{case}.s{s}.w'], rtol=1e-5, atol=1e-6)
        np.testing.assert_allclose(b.cpu().numpy(), g[f'c{case}.s{s}.b'], rtol=1e-5, atol=1e-6)
        np.testing.assert_allclose(ms[0].cpu().numpy(), g[f'c{case}.s{s}.m_w'], rtol=1e-5, atol=1e-9)
        np.testing.assert_allclose(vs[0].cpu().numpy(), g[f'c{case}.s{s}.v_w'], rtol=1e-5, atol=1e-12)
    assert ops.device_error() == 0


def test_forward_into_zero_padded_buffer_skips_the_padding():
    """`y_pad_zero = 1`: the forward writes only each member's block, rounded up to 32
    columns (the caller states that y's padding already holds zeros).  Into a zeroed buffer the
    result equals the normal forward bit for bit; a sentinel planted in the padding past that is
    left as it is."""
    import ctypes

    from tabpack_b200 import _lib, ops

    P, B, K, N = 6, 640, 256, 520
    rng = np.random.default_rng(8)
    out_np = (rng.integers(2, 66, P) * 8).astype(np.int32)
    outf = torch.from_numpy(out_np).cuda()
    p = torch.from_numpy(rng.uniform(0, 0.5, P).astype(np.float32)).cuda()
    g = torch.Generator(device='cuda').manual_seed(8)
    x = torch.randn(P, B, K, device='cuda', generator=g).bfloat16()
    w = (torch.randn(P, N, K, device='cuda', generator=g) / 16).bfloat16()
    b = torch.randn(P, N, device='cuda', generator=g) / 16
    kw = dict(out_features=outf, relu=True, dropout_p=p, seed=3, offset=1)
    want = ops.linear_forward(x, w, b, **kw)
    lib = _lib.load()
    col = torch.arange(N, device='cuda')[None, None, :]
    pad = col >= outf[:, None, None]
    far = col >= ((outf[:, None, None] + 31) // 32) * 32  # beyond the chunk that holds the last column
    for fill in (0.0, 7.0):
        y = torch.zeros(P, B, N, device='cuda', dtype=torch.bfloat16).masked_fill_(pad, fill)
        a = _lib.LinearArgs()
        a.P, a.B, a.max_in, a.max_out, a.dtype = P, B, K, N, _lib.TP_DTYPE_BF16
        a.out_features, a.relu, a.dropout_p, a.seed, a.offset = outf.data_ptr(), 1, p.data_ptr(), 3, 1
        a.x, a.w, a.bias, a.y, a.y_pad_zero = x.data_ptr(), w.data_ptr(), b.data_ptr(), y.data_ptr(), 1
        assert lib.tp_linear_forward(ctypes.byref(a), torch.cuda.current_stream().cuda_stream) == 0
        torch.cuda.synchronize()
        assert torch.equal(y[~pad.expand_as(y)].view(torch.int16), want[~pad.expand_as(want)].view(torch.int16))
        assert bool((y[far.expand_as(y)] == fill).all())
        assert bool((y[(pad & ~far).expand_as(y)] == 0).all())


@pytest.mark.parametrize('B', [1000, 258])
def test_gathered_input_matches_the_materialised_batch(B):
    """The first layer with its batch gathered by the GEMMs' operand loads (a (rows, 2544)
    bf16 table and per-member row indices, TMA gather4) against the same layer on the
    materialised per-member batch table[row_index]: forward output (ReLU + dropout, ragged
    widths), weight and bias gradients.  Rows past the batch (B not a multiple of the tiles)
    included."""
    from tabpack_b200 import ops

    P, N, K, O = 12, 4099, 2544, 1024
    rng = np.random.default_rng(B)
    out_np = (rng.integers(16, 129, P) * 8).astype(np.int32)
    outf = torch.from_numpy(out_np).cuda()
    inf = torch.full((P,), 2538, dtype=torch.int32, device='cuda')
    p = torch.from_numpy(rng.uniform(0, 0.5, P).astype(np.float32)).cuda()
    g = torch.Generator(device='cuda').manual_seed(B)
    kin = torch.arange(K, device='cuda') < 2538
    table = (torch.randn(N, K, device='cuda', generator=g) * kin).bfloat16()
    ri = torch.randint(0, N, (P, B), device='cuda', generator=g)
    w = ((torch.rand(P, O, K, device='cuda', generator=g) * 2 - 1) / 50 * kin).bfloat16()
    b = (torch.rand(P, O, device='cuda', generator=g) * 2 - 1) / 50
    kw = dict(in_features=inf, out_features=outf, relu=True, dropout_p=p, seed=11, offset=2)
    x = table[ri]  # (P, B, K) materialised
    y_g = ops.linear_forward(table, w, b, row_index=ri, **kw)
    y_m = ops.linear_forward(x, w, b, **kw)
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    _close_dev(y_g, y_m, BF16_RTOL, 'gathered forward')
    print('forward: bit-equal fraction', float((y_g.view(torch.int16) == y_m.view(torch.int16)).float().mean()))
    dy = torch.randn(P, B, O, device='cuda', generator=g).bfloat16()
    _, dw_g, db_g = ops.linear_backward(dy, table, w, y_g, row_index=ri, need_dx=False, **kw)
    _, dw_m, db_m = ops.linear_backward(dy, x, w, y_m, need_dx=False, **kw)
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    _close_dev(db_g, db_m, 1e-4, 'gathered bias gradient')
    _close_dev(dw_g, dw_m, BF16_RTOL, 'gathered weight gradient')
    pad = torch.arange(O, device='cuda')[None, :, None] >= outf[:, None, None]
    assert int(torch.count_nonzero(dw_g * pad)) == 0
    print('weight gradient: bit-equal fraction', float((dw_g == dw_m).float().mean()))
