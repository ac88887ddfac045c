"""Packed linear / block / MLP-backbone forward and backward (numpy restatement).

TEST INFRASTRUCTURE ONLY (see `oracle/__init__.py`).

Shapes follow the reference's pack convention (`PACK_DIM = 0`, `BATCH_DIM = 1`,
`src/tabpackage/nn.py:29-30`): activations are padded `(P, B, max_width)`,
weights `(P, max_out, max_in)`, biases `(P, max_out)`, and per-member widths
are `(P,)` arrays.  All arithmetic runs in the dtype of the inputs (float32 to
mirror the reference's fp32 mode, float64 for ground truth).
"""

from __future__ import annotations

import numpy as np

from oracle.philox import dropout_keep_mask, keep_scale


def col_mask(widths, max_width: int, dtype) -> np.ndarray:
    """(P, 1, max_width) 0/1 mask of columns below each member's width.

    Follows the output mask of `LinearPack.forward` (`nn.py:810-815`).
    """
    widths = np.asarray(widths)
    m = np.arange(max_width)[None, :] < widths[:, None]
    return m.astype(dtype)[:, None, :]


def expand_input(x: np.ndarray, pack_size: int) -> np.ndarray:
    """`PackView.forward` (`nn.py:88-89`): a 2-D input is shared by all members."""
    if x.ndim == 2:
        return np.broadcast_to(x[None], (pack_size, *x.shape))
    return x


def linear_forward(x, weight, bias, out_features=None):
    """`LinearPack.forward` (`nn.py:792-816`): `baddbmm(b, x, W^T)` then out mask."""
    P = weight.shape[0]
    x = expand_input(x, P)
    y = np.matmul(x, np.swapaxes(weight, -1, -2))
    if bias is not None:
        y = y + bias[:, None, :]
    if out_features is not None:
        y = y * col_mask(out_features, weight.shape[1], y.dtype)
    return y


def linear_backward(x, weight, out_features, dy):
    """Autograd of `linear_forward`: returns (dx, dW, db).

    dx keeps the reference's padded semantics: columns at or beyond a member's
    `in_features` get `dy @ W` of the (random) pad weights.
    """
    P = weight.shape[0]
    x = expand_input(x, P)
    if out_features is not None:
        dy = dy * col_mask(out_features, weight.shape[1], dy.dtype)
    dx = np.matmul(dy, weight)
    dW = np.matmul(np.swapaxes(dy, -1, -2), x)
    db = dy.sum(axis=1)
    return dx, dW, db


def dropout_mask_values(*, seed, offset, members, n_rows, n_cols, p, dtype):
    """The tensor `mask.div_(p_keep)` of `DropoutPack.forward` (`nn.py:897-901`)
    with the Bernoulli draw replaced by the Philox keep mask."""
    keep = dropout_keep_mask(
        seed=seed, offset=offset, members=members, n_rows=n_rows, n_cols=n_cols, p=p
    )
    scale = keep_scale(p).astype(dtype)
    return keep.astype(dtype) * scale[:, None, None]


def block_forward(x, weight, bias, out_features, *, mask_values=None, relu=True):
    """`MLPBackbonePack.Block.forward` (`nn.py:1071-1079`): Linear -> ReLU -> Dropout.

    `mask_values` is the (P, B, max_out) tensor `mask / p_keep` (None = eval mode
    or p = 0).  Returns (y, pre) where `pre` is the masked linear output.
    """
    pre = linear_forward(x, weight, bias, out_features)
    a = np.maximum(pre, 0) if relu else pre
    y = a if mask_values is None else mask_values * a
    return y, pre


def block_backward(x, weight, out_features, pre, dy, *, mask_values=None, relu=True):
    """Autograd of `block_forward`: returns (dx, dW, db)."""
    g = dy if mask_values is None else dy * mask_values
    if relu:
        g = g * (pre > 0).astype(g.dtype)
    return linear_backward(x, weight, out_features, g)


def mlp_forward_dense(x, blocks, n_blocks=None, *, masks=None, relu=True):
    """`MLPBackbonePack._forward_dense` (`nn.py:1272-1288`).

    `blocks` is a list of (weight, bias, out_features); members with
    `n_blocks <= i` keep their previous activation (`torch.where`).  Returns the
    output and the per-block cache needed by `mlp_backward_dense`.
    """
    cache = []
    for i, (w, b, of) in enumerate(blocks):
        mv = None if masks is None else masks[i]
        x_in = expand_input(x, w.shape[0])
        y, pre = block_forward(x_in, w, b, of, mask_values=mv, relu=relu)
        if n_blocks is not None and i > 0:
            active = (np.asarray(n_blocks) > i)[:, None, None]
            y = np.where(active, y, x_in)
        cache.append((x_in, pre, mv))
        x = y
    return x, cache


def mlp_backward_dense(blocks, cache, dy, n_blocks=None, *, relu=True):
    """Autograd of `mlp_forward_dense`: returns (dx, [(dW, db), ...])."""
    grads = [None] * len(blocks)
    for i in range(len(blocks) - 1, -1, -1):
        w, b, of = blocks[i]
        x_in, pre, mv = cache[i]
        if n_blocks is not None and i > 0:
            active = (np.asarray(n_blocks) > i)[:, None, None]
            dy_block = np.where(active, dy, 0)
            dy_pass = np.where(active, 0, dy)
        else:
            dy_block, dy_pass = dy, 0
        dx, dW, db = block_backward(x_in, w, of, pre, dy_block, mask_values=mv, relu=relu)
        grads[i] = (dW, db)
        dy = dx + dy_pass
    return dy, grads


def one_hot_encode(x_cat: np.ndarray, cardinalities, dtype) -> np.ndarray:
    """`_OneHotEncoding.forward` (`nn.py:1853-1871`): the value `card` (unknown
    category) encodes as all zeros."""
    parts = []
    for j, card in enumerate(cardinalities):
        v = x_cat[..., j]
        oh = (v[..., None] == np.arange(card)[None]).astype(dtype)
        parts.append(oh)
    return np.concatenate(parts, axis=-1)


def cosine_embeddings_forward(x, weight, bias, aw, ab, d_embedding=None):
    """`CosineEmbeddingsPack.forward` (`nn.py:1783-1833`), concat_input=True.

    x (P, B, F); weight, bias (P, F, D-1); aw, ab (P, F, D) (the elementwise affine);
    d_embedding (P,) or None.  out[..., 0] = ab0 + aw0 x, out[..., k] = ab_k + aw_k
    cos(2 pi b_{k-1} + 2 pi w_{k-1} x), with aw, ab zero at k >= d_embedding.  The
    factor 2 pi multiplies the parameters in their own dtype (`weight * (2 * torch.pi)`).
    Returns (y (P, B, F, D), cache).
    """
    dt = x.dtype
    D = aw.shape[-1]
    mask = None
    if d_embedding is not None:
        mask = (np.arange(D)[None] < np.asarray(d_embedding)[:, None]).astype(dt)[:, None, :]
        aw, ab = aw * mask, ab * mask
    two_pi = dt.type(2 * np.pi)
    w2, b2 = weight * two_pi, bias * two_pi
    z = b2[:, None] + w2[:, None] * x[..., None]
    cat = np.concatenate([x[..., None], np.cos(z)], -1)
    y = ab[:, None] + aw[:, None] * cat
    return y, (x, z, cat, aw, mask)


def cosine_embeddings_backward(cache, dy):
    """Autograd of `cosine_embeddings_forward` w.r.t. (weight, bias, aw, ab)."""
    x, z, cat, aw_m, mask = cache
    two_pi = x.dtype.type(2 * np.pi)
    dab = dy.sum(1)
    daw = (dy * cat).sum(1)
    if mask is not None:
        dab, daw = dab * mask, daw * mask
    dz = (dy * aw_m[:, None])[..., 1:] * -np.sin(z)
    dweight = (dz * x[..., None]).sum(1) * two_pi
    dbias = dz.sum(1) * two_pi
    return dweight, dbias, daw, dab
