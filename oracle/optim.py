"""AdamW / Muon optimizer-pack steps and Newton-Schulz (numpy restatement).

TEST INFRASTRUCTURE ONLY (see `oracle/__init__.py`).

Hyperparameters are either Python floats (shared by all members) or `(P,)`
float32 arrays (per member), exactly like the group values of
`OptimizerPack` (`src/tabpackage/optim.py:92-117`).  `bf16_round` emulates
round-to-nearest-even to bfloat16 so that the bf16 Newton-Schulz iteration
(`optim.py:464-490`) can be restated on the CPU.
"""

from __future__ import annotations

import numpy as np

F32 = np.float32


def bf16_round(x) -> np.ndarray:
    """Round float32 values to the nearest bfloat16 (ties to even), as float32."""
    x = np.asarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    bias = ((u >> np.uint64(16)) & np.uint64(1)) + np.uint64(0x7FFF)
    r = ((u + bias) & np.uint64(0xFFFF0000)).astype(np.uint32)
    out = r.view(np.float32).copy()
    nan = np.isnan(x)
    if nan.any():
        out[nan] = np.float32(np.nan)
    return out


def _bcast(v, ndim):
    """`_maybe_unsqueeze` (`optim.py:250-266`)."""
    if isinstance(v, np.ndarray):
        return v.reshape(v.shape[0], *([1] * (ndim - 1)))
    return v


def lerp(a, b, w):
    """torch's `lerp`: `a + w*(b-a)` if |w| < 0.5 else `b - (b-a)*(1-w)` (fp32)."""
    a = np.asarray(a, dtype=F32)
    b = np.asarray(b, dtype=F32)
    w = np.asarray(w, dtype=F32)
    small = np.abs(w) < F32(0.5)
    d = (b - a).astype(F32)
    lo = (a + (w * d).astype(F32)).astype(F32)
    hi = (b - (d * (F32(1) - w).astype(F32)).astype(F32)).astype(F32)
    return np.where(small, lo, hi).astype(F32)


def wd_multiplier(lr, wd):
    """`_make_weight_decay_multiplier` (`optim.py:240-247`)."""
    if (isinstance(lr, float) and lr == 0.0) or (isinstance(wd, float) and wd == 0.0):
        return None
    if isinstance(lr, float) and isinstance(wd, float):
        return 1 - lr * wd
    return (F32(1) - (np.asarray(lr, F32) * np.asarray(wd, F32)).astype(F32)).astype(F32)


def adamw_step(p, g, state, *, lr, beta1, beta2, eps, weight_decay, support_replacement):
    """One `AdamWPack.step` for one parameter pack (`optim.py:347-427`).

    `state` is a dict with 'step' (int or (P,) int64), 'exp_avg', 'exp_avg_sq';
    missing keys are initialised as in `optim.py:370-390`.  Updates in place and
    returns `p`.
    """
    nd = p.ndim
    if not state:
        state['step'] = np.zeros(p.shape[0], np.int64) if support_replacement else 0
        state['exp_avg'] = np.zeros_like(p)
        state['exp_avg_sq'] = np.zeros_like(p)
    m, v = state['exp_avg'], state['exp_avg_sq']
    state['step'] = state['step'] + 1
    step = state['step']

    mult = wd_multiplier(lr, weight_decay)
    if mult is not None:
        p[...] = (p * _bcast(np.asarray(mult, F32) if isinstance(mult, np.ndarray) else F32(mult), nd)).astype(F32)

    one_m_b1 = (1 - beta1) if isinstance(beta1, float) else (F32(1) - beta1).astype(F32)
    m[...] = lerp(m, g, _bcast(np.asarray(one_m_b1, F32), nd) if isinstance(one_m_b1, np.ndarray) else F32(one_m_b1))
    if isinstance(beta2, float):
        v[...] = (v * F32(beta2)).astype(F32)
        v[...] = (v + ((F32(1 - beta2) * g).astype(F32) * g).astype(F32)).astype(F32)
    else:
        w2 = (F32(1) - beta2).astype(F32)
        v[...] = lerp(v, (g * g).astype(F32), _bcast(w2, nd))

    def pow_(base, e):
        if isinstance(base, float) and isinstance(e, (int, np.integer)):
            return base ** int(e)
        return np.power(np.asarray(base, F32), np.asarray(e)).astype(F32)

    bc1 = pow_(beta1, step)
    bc1 = (1 - bc1) if isinstance(bc1, float) else (F32(1) - bc1).astype(F32)
    bc2 = pow_(beta2, step)
    bc2 = (1 - bc2) if isinstance(bc2, float) else (F32(1) - bc2).astype(F32)
    step_size = lr / bc1 if isinstance(lr, float) and isinstance(bc1, float) else (np.asarray(lr, F32) / np.asarray(bc1, F32)).astype(F32)

    if isinstance(bc2, float):
        denom = (np.sqrt(v).astype(F32) / F32(bc2 ** 0.5)).astype(F32)
    else:
        denom = (np.sqrt(v).astype(F32) / _bcast(np.sqrt(bc2).astype(F32), nd)).astype(F32)
    denom = (denom + (_bcast(eps, nd) if isinstance(eps, np.ndarray) else F32(eps))).astype(F32)

    if isinstance(step_size, float):
        p[...] = (p + (F32(-step_size) * m).astype(F32) / denom).astype(F32)
    else:
        upd = ((m / denom).astype(F32) * _bcast(step_size, nd)).astype(F32)
        p[...] = (p - upd).astype(F32)
    return p


def muon_update_scale(out_features, in_features, max_out, max_in):
    """`compute_muon_update_scale_pack` (`optim.py:430-453`)."""
    if out_features is None and in_features is None:
        return None
    P = len(out_features if out_features is not None else in_features)
    o = np.full(P, max_out, F32) if out_features is None else np.asarray(out_features, F32)
    i = np.full(P, max_in, F32) if in_features is None else np.asarray(in_features, F32)
    return np.sqrt(np.maximum((o / i).astype(F32), F32(1))).astype(F32)


NS_COEFFS = (3.4445, -4.7750, 2.0315)


def _bf16_mm(a, b):
    """bf16 x bf16 -> fp32 accumulate (values already bf16-representable)."""
    return np.matmul(a.astype(F32), b.astype(F32)).astype(F32)


def newton_schulz5(G, steps: int = 5):
    """`_zeropower_via_newtonschulz5` (`optim.py:464-490`) with bf16 emulation.

    G: (P, r, c).  Every tensor op rounds its result to bf16 once; matmuls
    accumulate in fp32 and apply `baddbmm`'s alpha/beta before rounding.
    """
    a, b, c = (F32(x) for x in NS_COEFFS)
    X = bf16_round(G)
    transposed = G.shape[-2] > G.shape[-1]
    if transposed:
        X = np.swapaxes(X, -1, -2)
    nrm = bf16_round(np.sqrt(np.sum((X.astype(np.float64)) ** 2, axis=(-2, -1), keepdims=True)).astype(F32))
    den = bf16_round((nrm + F32(1e-7)).astype(F32))
    X = bf16_round((X / den).astype(F32))
    for _ in range(steps):
        A = bf16_round(_bf16_mm(X, np.swapaxes(X, -1, -2)))
        B = bf16_round((b * A + c * _bf16_mm(A, A)).astype(F32))
        X = bf16_round((a * X + _bf16_mm(B, X)).astype(F32))
    if transposed:
        X = np.swapaxes(X, -1, -2)
    return X


def newton_schulz5_ragged(G, out_features, in_features, steps: int = 5):
    """Newton-Schulz on each member's real `(out_i, in_i)` block, oriented so
    that the Gram matrix is `min(out_i, in_i)` square; pads stay exactly zero.

    In exact arithmetic this equals `newton_schulz5` on the zero-padded pack
    (the quintic map commutes with zero padding and with transposition); in
    bf16 the two differ only by rounding.
    """
    out = np.zeros_like(G, dtype=F32)
    for i in range(G.shape[0]):
        o, n = int(out_features[i]), int(in_features[i])
        blk = G[i : i + 1, :o, :n]
        out[i, :o, :n] = newton_schulz5(blk, steps)[0]
    return out


def muon_step(p, g, state, *, lr, momentum, weight_decay, nesterov, update_scale,
              ns_steps=5, ns_fn=None):
    """One Muon group step of `MuonAdamWPack._step_muon` (`optim.py:682-774`)
    for a single `(P, out, in)` parameter pack.  Updates p, g (Nesterov mutates
    the gradient in place, `allow_inplace_grad_mutation=True`) and the state."""
    nd = p.ndim
    if not state:
        state['muon_momentum_buffer'] = np.zeros_like(p)
    mb = state['muon_momentum_buffer']
    mult = wd_multiplier(lr, weight_decay)
    if mult is not None:
        p[...] = (p * _bcast(np.asarray(mult, F32) if isinstance(mult, np.ndarray) else F32(mult), nd)).astype(F32)
    one_m_mu = (1 - momentum) if isinstance(momentum, float) else (F32(1) - momentum).astype(F32)
    mb[...] = lerp(mb, g, _bcast(np.asarray(one_m_mu, F32), nd) if isinstance(one_m_mu, np.ndarray) else F32(one_m_mu))
    if nesterov:
        g[...] = lerp(g, mb, _bcast(np.asarray(momentum, F32), nd) if isinstance(momentum, np.ndarray) else F32(momentum))
        upd_in = g
    else:
        upd_in = mb
    U = (ns_fn or newton_schulz5)(upd_in, ns_steps)
    if update_scale is None:
        scaled = lr * max(1, g.shape[-2] / g.shape[-1]) ** 0.5 if isinstance(lr, float) else (
            np.asarray(lr, F32) * F32(max(1, g.shape[-2] / g.shape[-1]) ** 0.5)).astype(F32)
    else:
        scaled = (np.asarray(lr, F32) * update_scale).astype(F32) if isinstance(lr, np.ndarray) else (F32(lr) * update_scale).astype(F32)
    if isinstance(scaled, float):
        p[...] = (p + F32(-scaled) * U).astype(F32)
    else:
        p[...] = (p - (U * _bcast(scaled, nd)).astype(F32)).astype(F32)
    return p
