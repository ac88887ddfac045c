"""Member-sharded training and prediction on the B200 hot path.

`PackTrainer` runs the per-step loop of `tabpackage.train`'s `_train`
(`src/tabpackage/_training.py:2643-2692`) -- shuffled per-member batches, forward,
per-member losses summed, backward, optimizer-pack step -- and the per-epoch
evaluation + greedy ensemble update (`_training.py:2697-2831`) with members sharded
over the GPUs of one box.  Everything that depends on randomness is keyed by global
member id (initialisation, batch order, dropout), so a member trains identically on
1, 2, 4 or 8 GPUs.  `PackPredictor` is the inference side of `TabPackPredictor`
(`_training.py:1909-2018`): every member's transformed prediction plus ensemble heads
that average selected members, summed across ranks with one all-reduce.

The reference's checkpoint store, early stopping and model-replacement queue are host
bookkeeping around this loop and are not part of this module.
"""

from __future__ import annotations

import dataclasses

import torch
import torch.distributed as dist
import torch.nn.functional as F
from torch import Tensor

from tabpack_b200 import ops
from tabpack_b200.ensemble import greedy_ensemble
from tabpack_b200.metrics import PackScore
from tabpack_b200.nn import CosineEmbeddingsPack, LinearPack, TabPack
from tabpack_b200.optim import AdamWPack, MuonAdamWPack, split_weight_decay
from tabpack_b200.shard import allreduce_sum_, gather_members, member_ranges

_LOSSES = ('mse', 'bce', 'ce')


def _mix(*xs: int) -> int:
    """64-bit mixing of integers (splitmix64 steps) for per-member generator seeds."""
    h = 0x9E3779B97F4A7C15
    for x in xs:
        h = (h ^ (x & 0xFFFFFFFFFFFFFFFF)) * 0xBF58476D1CE4E5B9 & 0xFFFFFFFFFFFFFFFF
        h ^= h >> 31
    return h & 0x7FFFFFFFFFFFFFFF


@torch.no_grad()
def init_member_parameters_(model: torch.nn.Module, *, seed: int, member_ids: list[int]) -> None:
    """Re-initialise every LinearPack (and CosineEmbeddingsPack) member from its own generator.

    Same distribution as `LinearPack.reset_parameters` (`nn.py:702-747`), U(+-1/sqrt(in_i))
    for weights and biases, but member m of the j-th LinearPack draws from a generator
    seeded by (seed, global member id, j): initial weights do not depend on sharding.
    """
    for j, emb in enumerate(m for m in model.modules() if isinstance(m, CosineEmbeddingsPack)):
        # CosineEmbeddingsPack.reset_parameters (`nn.py:1706-1753`): truncated N(0, 1) on
        # [-3, 3] times the member's init scale, the affine parts zero
        for m, gid in enumerate(member_ids):
            g = torch.Generator(device=emb.weight.device).manual_seed(_mix(seed, gid, 0xE0 + j))
            w = torch.empty(emb.weight.shape[1:], device=emb.weight.device, dtype=emb.weight.dtype)
            torch.nn.init.trunc_normal_(w, a=-3.0, b=3.0, generator=g)
            scale = emb.init_scale if isinstance(emb.init_scale, float) else float(emb.init_scale[m])
            emb.weight[m].copy_(w * scale)
            for p in (emb.bias, emb.elementwise_affine_weight, emb.elementwise_affine_bias):
                p[m].zero_()
    linears = [m for m in model.modules() if isinstance(m, LinearPack)]
    for j, lin in enumerate(linears):
        inf = lin.in_features.tolist() if lin.in_features is not None else [lin.max_in_features] * lin.pack_size
        for m, gid in enumerate(member_ids):
            g = torch.Generator(device=lin.weight.device).manual_seed(_mix(seed, gid, j))
            b = inf[m] ** -0.5
            for p in (lin.weight, lin.bias):
                if p is None:
                    continue
                u = torch.rand(p.shape[1:], generator=g, device=p.device, dtype=p.dtype)
                p[m].copy_(torch.lerp(torch.full_like(u, -b), torch.full_like(u, b), u))


def _transpose(per_member: list[dict]) -> dict:
    """`transpose_dicts_recursively` (`_training.py:66-101`) for flat/nested dicts."""
    out: dict = {}
    for k in per_member[0]:
        v0 = per_member[0][k]
        if isinstance(v0, dict):
            out[k] = _transpose([d[k] for d in per_member])
        else:
            out[k] = [d[k] for d in per_member]
    return out


def _merge(base: dict, update: dict) -> dict:
    """`base` with `update` merged in, nested dicts (e.g. `numerical_embeddings`) key by key."""
    out = dict(base)
    for k, v in update.items():
        out[k] = _merge(out[k], v) if isinstance(v, dict) and isinstance(out.get(k), dict) else v
    return out


def member_loss(loss: str, y_pred: Tensor, y: Tensor) -> Tensor:
    """Per-member training loss (P,) from raw outputs (P, B, d_out) and labels (P, B)."""
    if loss == 'mse':
        return ((y_pred[..., 0] - y) ** 2).mean(1)
    if loss == 'bce':
        return F.binary_cross_entropy_with_logits(y_pred[..., 0], y.float(), reduction='none').mean(1)
    if loss == 'ce':
        return F.cross_entropy(y_pred.transpose(1, 2), y, reduction='none').mean(1)
    raise ValueError(f'unknown loss {loss!r}')


def transform(loss: str, y_pred: Tensor) -> Tensor:
    """Prediction transform: identity (regression), sigmoid (binary), softmax (multiclass)."""
    if loss == 'mse':
        return y_pred[..., 0]
    if loss == 'bce':
        return torch.sigmoid(y_pred[..., 0])
    return ops.softmax_rows(y_pred)


@dataclasses.dataclass
class EpochResult:
    epoch: int
    train_loss: Tensor            # (P_total,) mean per-member training loss of the epoch
    val_metric: Tensor            # (P_total,) per-member validation metric
    ensemble_idx: Tensor          # global member ids selected by greedy ensembling
    ensemble_weights: Tensor | None
    ensemble_score: float         # the ensemble's validation metric


class PackTrainer:
    """Trains a pack of TabPack MLPs, members sharded over the process group."""

    def __init__(self, *, n_members: int, model: dict, per_member_model: list[dict], optimizer: dict,
                 per_member_optimizer: list[dict] | None = None, loss: str, seed: int, device,
                 autocast_bf16: bool = True, group=None, cost: list[float] | None = None,
                 member_range: tuple[int, int] | None = None) -> None:
        """`member_range` pins this trainer to global members [lo, hi) without a process
        group (several shards on one device); otherwise the group's rank picks its range."""
        if loss not in _LOSSES:
            raise ValueError(f'loss must be one of {_LOSSES}')
        self.group = group
        self.world = dist.get_world_size(group) if (dist.is_initialized() and member_range is None) else 1
        self.rank = dist.get_rank(group) if (dist.is_initialized() and member_range is None) else 0
        self.ranges = member_ranges(n_members, self.world, cost)
        if member_range is None:
            self._check_ranges(self.ranges)
        lo, hi = self.ranges[self.rank] if member_range is None else member_range
        if hi <= lo:
            raise ValueError('every rank needs at least one member')
        self.lo, self.hi = lo, hi
        self.counts = [b - a for a, b in self.ranges] if member_range is None else [hi - lo]
        self.loss = loss
        self.seed = int(seed)
        self.autocast = autocast_bf16
        self.device = torch.device(device)
        local = per_member_model[lo:hi]
        kw = _merge(model, _transpose(local))
        self.model = TabPack(pack_size=hi - lo, **kw).to(self.device)
        self.model.backbone.set_member_base(lo)
        self.model.backbone._stream.seed = _mix(self.seed, 0xD0)  # one Philox key on every rank
        init_member_parameters_(self.model, seed=self.seed, member_ids=list(range(lo, hi)))
        okw = dict(optimizer)
        otype = okw.pop('type')
        if per_member_optimizer is not None:
            okw.update(_transpose(per_member_optimizer[lo:hi]))
        if otype == 'muon':
            groups = [MuonAdamWPack.make_muon_parameter_group(b.linear) for b in self.model.backbone.blocks]
            muon_params = {id(g['params'][0]) for g in groups}
            decay, no_decay = split_weight_decay(self.model)
            groups.append({'params': [p for p in no_decay if id(p) not in muon_params], 'weight_decay': 0.0})
            groups.append({'params': [p for p in decay if id(p) not in muon_params]})
            self.opt = MuonAdamWPack(groups, pack_size=hi - lo, allow_inplace_grad_mutation=True, **okw)
        elif otype == 'adamw':
            wd, nd = split_weight_decay(self.model)
            self.opt = AdamWPack([{'params': nd, 'weight_decay': 0.0}, {'params': wd}], pack_size=hi - lo, **okw)
        else:
            raise ValueError("optimizer type must be 'muon' or 'adamw'")

    @staticmethod
    def _check_ranges(ranges: list[tuple[int, int]]) -> None:
        """Every rank computes the same ranges, so all ranks raise together here, before
        any collective, instead of one rank leaving the others waiting in one."""
        if any(b <= a for a, b in ranges):
            raise ValueError(f'every rank needs at least one member ({ranges[-1][1]} members over '
                             f'{len(ranges)} ranks)')

    # ------------------------------------------------------------------ training
    def _batches(self, n_rows: int, batch_size: int, epoch: int):
        keys = ops.permutation_keys(seed=_mix(self.seed, 0xBA), epoch=epoch, member_base=self.lo,
                                    P=self.hi - self.lo, N=n_rows, device=self.device)
        order = torch.argsort(keys, dim=1, stable=True)
        return order.split(batch_size, dim=1)

    def fit_epoch(self, data: dict, *, batch_size: int, epoch: int) -> Tensor:
        """One epoch over `data` ({'x_num', 'x_cat', 'y'} on this device); returns the
        mean training loss of every member (P_total,) (gathered when sharded)."""
        self.model.train()
        n = len(data['y'])
        total = torch.zeros(self.hi - self.lo, device=self.device)
        steps = 0
        for idx in self._batches(n, batch_size, epoch):
            y = data['y'][idx]
            with torch.autocast('cuda', dtype=torch.bfloat16, enabled=self.autocast):
                # the batch gather runs inside the first-layer input build where it can
                out = self.model.forward_rows(data.get('x_num'), data.get('x_cat'), idx)
            losses = member_loss(self.loss, out.float(), y)
            losses.sum().backward()
            self.opt.step()
            self.opt.zero_grad()
            total += losses.detach()
            steps += 1
        mean = total / max(steps, 1)
        return gather_members(mean, self.counts, self.group) if self.world > 1 else mean

    # ------------------------------------------------------------------ evaluation
    @torch.no_grad()
    def predict_local(self, data: dict, *, eval_batch_size: int = 32768, member_chunk: int | None = None) -> Tensor:
        """Transformed predictions of this rank's members on a shared dataset.  `member_chunk`
        runs the members in groups of that size (bounds the activations of wide packs on large
        batches: each group is a `pack_idx` selection of the pack)."""
        self.model.eval()
        n = len(data['y']) if 'y' in data else len(next(iter(data.values())))
        P = self.hi - self.lo
        chunks = [None] if member_chunk is None or member_chunk >= P else [
            torch.arange(c, min(P, c + member_chunk), device=self.device) for c in range(0, P, member_chunk)]
        parts = []
        for i in range(0, n, eval_batch_size):
            xn = data['x_num'][i: i + eval_batch_size] if 'x_num' in data else None
            xc = data['x_cat'][i: i + eval_batch_size] if 'x_cat' in data else None
            outs = []
            for idx in chunks:
                with torch.no_grad(), torch.autocast('cuda', dtype=torch.bfloat16, enabled=self.autocast):
                    out = self.model(xn, xc, idx)
                outs.append(transform(self.loss, out.float()))
            parts.append(outs[0] if len(outs) == 1 else torch.cat(outs, 0))
        return torch.cat(parts, 1)

    def _score(self, y_val: Tensor) -> PackScore:
        return PackScore({'mse': 'mse', 'bce': 'bce', 'ce': 'ce'}[self.loss], y_val, maximize=False)

    def evaluate_and_ensemble(self, data: dict, *, epoch: int, train_loss: Tensor, eval_batch_size: int = 32768,
                              max_ensemble_size: int | None = 32) -> EpochResult:
        """Validation predictions of all members (all-gathered over NVLink when sharded),
        per-member metrics and a greedy ensemble built from them."""
        local = self.predict_local(data, eval_batch_size=eval_batch_size)
        preds = gather_members(local, self.counts, self.group) if self.world > 1 else local
        score = self._score(data['y'])
        metric = -score(preds)
        idx, w = greedy_ensemble(preds, score_fn=score, max_ensemble_size=max_ensemble_size)
        ens = preds[idx].mean(0, keepdim=True)
        ens_score = float(-score(ens)[0])
        return EpochResult(epoch, train_loss, metric, idx, w, ens_score)


class PackPredictor(torch.nn.Module):
    """Inference over a (sharded) pack: every member's transformed prediction and ensemble
    heads averaging the selected global members (`_training.py:1909-2018`)."""

    def __init__(self, trainer: PackTrainer, ensembles: dict[str, Tensor]) -> None:
        super().__init__()
        self.trainer = trainer
        self.ensembles = {k: v.to(trainer.device, torch.int64) for k, v in ensembles.items()}

    @torch.no_grad()
    def forward(self, x_num: Tensor | None, x_cat: Tensor | None, *, eval_batch_size: int = 32768,
                member_chunk: int | None = None) -> tuple[Tensor, dict[str, Tensor]]:
        t = self.trainer
        data = {}
        if x_num is not None:
            data['x_num'] = x_num
        if x_cat is not None:
            data['x_cat'] = x_cat
        local = t.predict_local(data, eval_batch_size=eval_batch_size, member_chunk=member_chunk)  # (P_local, B[, C])
        flat = local.reshape(local.shape[0], -1).contiguous()
        heads = {}
        for name, gidx in self.ensembles.items():
            mine = gidx[(gidx >= t.lo) & (gidx < t.hi)] - t.lo
            part = torch.zeros(flat.shape[1], device=flat.device)
            if len(mine):
                part = ops.ensemble_mean(flat, mine.to(torch.int32)) * len(mine)
            if t.world > 1:
                allreduce_sum_(part, t.group)
            heads[name] = (part / len(gidx)).view(local.shape[1:])
        return local, heads


def assert_finite(x: Tensor, what: str) -> None:
    if not bool(torch.isfinite(x).all()):
        raise FloatingPointError(f'{what} is not finite')


__all__ = ['PackTrainer', 'PackPredictor', 'EpochResult', 'init_member_parameters_', 'member_loss', 'transform',
           'assert_finite']
