"""The reference's TabPack training step on the CPU, restated with the reference's own ops.

TEST INFRASTRUCTURE ONLY (see `oracle/__init__.py`): `bench.py` times it as the CPU
baseline of the full-training workload (its `cpu_baseline` leg and `--impl reference`).
Nothing in `tabpack_b200` imports it.

The reference is pure Python on PyTorch, so its CPU path for this workload is a sequence of
ATen ops; this module issues the same ops in the same order on CPU tensors:

* first-layer input: numerical features concatenated with the one-hot block
  (`_OneHotEncoding`, `src/tabpackage/nn.py:1836-1871`; `TabPack.forward`, `nn.py:2071-2107`);
* every block on every member, padded: `baddbmm` and the output-width mask
  (`LinearPack.forward`, `nn.py:792-816`), ReLU, dropout as `bernoulli_` / `p_keep`
  (`DropoutPack.forward`, `nn.py:886-903`), depth gating with `where`
  (`MLPBackbonePack._forward_dense`, `nn.py:1272-1288`); the output `LinearPack`;
* under bf16 autocast (`_training.py:154-167`), the outputs cast to fp32, per-member BCE with
  logits summed over members (`_training.py:2671-2682`), autograd backward;
* `MuonAdamWPack.step` (`optim.py:682-846`): decoupled weight decay, momentum `lerp_`,
  Nesterov blend, `_zeropower_via_newtonschulz5` in bf16 (`optim.py:464-490`), the update
  scaled by `compute_muon_update_scale_pack` (`optim.py:430-453`); AdamW for biases and the
  output layer.
"""

from __future__ import annotations

import numpy as np
import torch
import torch.nn.functional as F


def _newton_schulz(G: torch.Tensor, steps: int = 5) -> torch.Tensor:
    """`_zeropower_via_newtonschulz5` (`optim.py:464-490`)."""
    a, b, c = 3.4445, -4.7750, 2.0315
    X = G.bfloat16()
    tall = G.size(-2) > G.size(-1)
    if tall:
        X = X.mT
    X = X / (X.norm(dim=(-2, -1), keepdim=True) + 1e-7)
    for _ in range(steps):
        A = X @ X.mT
        B = torch.baddbmm(A, A, A, beta=b, alpha=c)
        X = torch.baddbmm(X, B, X, beta=a)
    return X.mT if tall else X


class TrainingStep:
    """A padded pack of TabPack MLPs (members of the full-training configuration) with
    Muon + AdamW, fp32 master parameters, bf16 autocast forward."""

    def __init__(self, *, n_num: int, cards: list[int], widths: list[int], depths: list[int], dropout: list[float],
                 max_width: int = 1024, max_depth: int = 4, seed: int = 0, adamw_lr: float = 1e-3,
                 muon_lr: float = 2e-2, weight_decay: float = 1e-5) -> None:
        g = torch.Generator().manual_seed(seed)
        P = len(widths)
        self.P, self.cards, self.max_depth = P, cards, max_depth
        self.d_in = n_num + sum(cards)
        self.width = torch.tensor(widths)
        self.depth = torch.tensor(depths)
        self.p = torch.tensor(dropout, dtype=torch.float32)
        self.W, self.b = [], []
        for j in range(max_depth):
            fan_in = self.d_in if j == 0 else max_width
            bound = (self.d_in if j == 0 else self.width.float()) ** -0.5
            bound = torch.as_tensor(bound, dtype=torch.float32).expand(P)
            w = (torch.rand(P, max_width, fan_in, generator=g) * 2 - 1) * bound[:, None, None]
            self.W.append(w.requires_grad_())
            self.b.append(((torch.rand(P, max_width, generator=g) * 2 - 1) * bound[:, None]).requires_grad_())
        hb = self.width.float() ** -0.5
        self.head_w = ((torch.rand(P, 1, max_width, generator=g) * 2 - 1) * hb[:, None, None]).requires_grad_()
        self.head_b = ((torch.rand(P, 1, generator=g) * 2 - 1) * hb[:, None]).requires_grad_()
        self.out_mask = (torch.arange(max_width)[None] < self.width[:, None]).float()
        self.muon_scale = [(torch.clamp(self.width.float() / (self.d_in if j == 0 else self.width.float()), min=1.0)
                            ).sqrt() for j in range(max_depth)]
        self.mom = [torch.zeros_like(w) for w in self.W]
        adam = self.b + [self.head_w, self.head_b]
        self.adam = [(t, torch.zeros_like(t), torch.zeros_like(t)) for t in adam]
        self.adamw_lr, self.muon_lr, self.wd = adamw_lr, muon_lr, weight_decay
        self.steps = 0

    def _input(self, x_num: torch.Tensor, x_cat: torch.Tensor) -> torch.Tensor:
        onehot = torch.cat([F.one_hot(x_cat[..., i], c + 1)[..., :-1] for i, c in enumerate(self.cards)], -1)
        return torch.cat([x_num, onehot.to(torch.get_default_dtype())], -1)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        for j in range(self.max_depth):
            y = torch.baddbmm(self.b[j].unsqueeze(1), x, self.W[j].transpose(-2, -1))
            y = y * self.out_mask.to(y.dtype).unsqueeze(1)
            y = torch.relu(y)
            keep = (1.0 - self.p)[:, None, None]
            mask = torch.empty_like(y).bernoulli_(keep.expand_as(y))
            y = mask.div_(keep) * y
            x = y if j == 0 else torch.where((j < self.depth).view(-1, 1, 1), y, x)
        return torch.baddbmm(self.head_b.unsqueeze(1), x, self.head_w.transpose(-2, -1))

    def step(self, x_num: torch.Tensor, x_cat: torch.Tensor, y: torch.Tensor) -> float:
        """One training step on a (P, B) batch of rows per member; returns the summed loss."""
        with torch.autocast('cpu', dtype=torch.bfloat16):
            out = self.forward(self._input(x_num, x_cat))
        losses = F.binary_cross_entropy_with_logits(out.float()[..., 0], y.float(), reduction='none').mean(1)
        loss = losses.sum()
        loss.backward()
        self.steps += 1
        with torch.no_grad():
            for j, w in enumerate(self.W):  # MuonAdamWPack._step_muon
                grad = w.grad
                w.mul_(1 - self.muon_lr * self.wd)
                self.mom[j].lerp_(grad, 1 - 0.95)
                update = grad.lerp_(self.mom[j], 0.95)
                update = _newton_schulz(update, 5)
                w.addcmul_(update.float(), (self.muon_lr * self.muon_scale[j])[:, None, None], value=-1)
                w.grad = None
            bc1, bc2 = 1 - 0.9 ** self.steps, 1 - 0.999 ** self.steps
            for t, m, v in self.adam:  # MuonAdamWPack._step_adamw
                grad = t.grad
                if t.ndim == 3:  # the output layer's weight takes weight decay, biases do not
                    t.mul_(1 - self.adamw_lr * self.wd)
                m.lerp_(grad, 1 - 0.9)
                v.mul_(0.999).addcmul_(grad, grad, value=1 - 0.999)
                denom = (v.sqrt() / bc2 ** 0.5).add_(1e-8)
                t.addcdiv_(m, denom, value=-self.adamw_lr / bc1)
                t.grad = None
        return float(loss.detach())


def sample_batch(rng: np.random.Generator, x_num: torch.Tensor, x_cat: torch.Tensor, y: torch.Tensor, P: int,
                 B: int):
    """A (P, B) batch of rows per member, as `v[batch_idx]` gathers it (`_training.py:2667-2669`)."""
    idx = torch.from_numpy(rng.integers(0, len(y), (P, B)))
    return x_num[idx], x_cat[idx], y[idx]


def block_step(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor, out_features: torch.Tensor, p: torch.Tensor,
               dy: torch.Tensor) -> torch.Tensor:
    """One `MLPBackbonePack.Block` forward and backward (`nn.py:1071-1079`) on the CPU in fp32 with
    the reference's ops: `baddbmm` + output-width mask (`LinearPack.forward`, `nn.py:792-816`),
    ReLU, `bernoulli_` dropout (`DropoutPack.forward`, `nn.py:886-903`), autograd for dx, dW, db.
    `x` (B, in) is shared by every member, as `PackView` expands it (`nn.py:84-99`)."""
    w = w.detach().requires_grad_()
    b = b.detach().requires_grad_()
    xs = x.detach().expand(w.shape[0], *x.shape).requires_grad_()
    y = torch.baddbmm(b.unsqueeze(1), xs, w.transpose(-2, -1))
    y = y * (torch.arange(w.shape[1])[None] < out_features[:, None]).to(y.dtype).unsqueeze(1)
    y = torch.relu(y)
    keep = (1.0 - p)[:, None, None]
    y = torch.empty_like(y).bernoulli_(keep.expand_as(y)).div_(keep) * y
    y.backward(dy)
    return y.detach()
