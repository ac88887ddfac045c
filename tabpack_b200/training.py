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

`PackTrainer.fit` runs the reference's epoch loop end to end (`_training.py:2643-2960`):
per-member best checkpoints by the validation metric with early-stopping patience
(`update_training_state`, `_training.py:754-821`), and an online greedy ensemble rebuilt
after every epoch from the current members, the best checkpoints of finished members and
the latest checkpoints of running ones, accepted only when its validation score improves
(`Ensemble.update`, `_training.py:1061-1183`).  With more models than pack slots
(`n_models`, the reference's `max_pack_size < n_models`), the slots of finished models take
the next model ids (`_training.py:2891-2927`, `pack_replace` `_training.py:860-924`) in one
global order that every rank computes alike (`shard.assign_replacements`).  A finished model
that no new model replaces keeps its slot with a zero learning rate (its parameters no longer
change) where the reference removes it from the pack.
"""

from __future__ import annotations

import dataclasses
import math
from typing import Callable

import torch
import torch.distributed as dist
import torch.nn.functional as F
from torch import Tensor

from tabpack_b200 import ops
from tabpack_b200.ensemble import compute_unsanitized_ensemble_predictions, greedy_ensemble
from tabpack_b200.metrics import PackScore
from tabpack_b200.nn import CosineEmbeddingsPack, LinearPack, TabPack
from tabpack_b200.optim import AdamWPack, MuonAdamWPack, split_weight_decay
from tabpack_b200.shard import allreduce_sum_, assign_replacements, gather_members, member_ranges

_LOSSES = ('mse', 'bce', 'ce')


def _mix(*xs: int) -> int:
    """64-bit mixing of integers (splitmix64 steps) for per-member generator seeds."""
    h = 0x9E3779B97F4A7C15
    for x in xs:
        h = (h ^ (x & 0xFFFFFFFFFFFFFFFF)) * 0xBF58476D1CE4E5B9 & 0xFFFFFFFFFFFFFFFF
        h ^= h >> 31
    return h & 0x7FFFFFFFFFFFFFFF


@torch.no_grad()
def init_member_parameters_(model: torch.nn.Module, *, seed: int, member_ids: list[int],
                            generator_device: str | torch.device | None = None,
                            pack_idx: list[int] | None = None) -> None:
    """Re-initialise every LinearPack (and CosineEmbeddingsPack) member from its own generator.

    Same distribution as `LinearPack.reset_parameters` (`nn.py:702-747`), U(+-1/sqrt(in_i))
    for weights and biases, but member m of the j-th LinearPack draws from a generator
    seeded by (seed, global member id, j): initial weights do not depend on sharding.
    The generators live on the parameters' device unless `generator_device` names another
    one (e.g. 'cpu': the same numbers on any machine, drawn on the host and copied over).
    `pack_idx` names the pack positions that take `member_ids` (default: 0, 1, ...).
    """
    slots = list(range(len(member_ids))) if pack_idx is None else list(pack_idx)
    if len(slots) != len(member_ids):
        raise ValueError('one pack position per member id is required')

    def gen(dev, key):
        d = torch.device(generator_device) if generator_device is not None else dev
        return torch.Generator(device=d).manual_seed(key), d

    for j, emb in enumerate(m for m in model.modules() if isinstance(m, CosineEmbeddingsPack)):
        # CosineEmbeddingsPack.reset_parameters (`nn.py:1706-1753`): truncated N(0, 1) on
        # [-3, 3] times the member's init scale, the affine parts zero
        for m, gid in zip(slots, member_ids):
            g, d = gen(emb.weight.device, _mix(seed, gid, 0xE0 + j))
            w = torch.empty(emb.weight.shape[1:], device=d, dtype=emb.weight.dtype)
            torch.nn.init.trunc_normal_(w, a=-3.0, b=3.0, generator=g)
            scale = emb.init_scale if isinstance(emb.init_scale, float) else float(emb.init_scale[m])
            emb.weight[m].copy_(w * scale)
            for p in (emb.bias, emb.elementwise_affine_weight, emb.elementwise_affine_bias):
                p[m].zero_()
    linears = [m for m in model.modules() if isinstance(m, LinearPack)]
    for j, lin in enumerate(linears):
        inf = lin.in_features.tolist() if lin.in_features is not None else [lin.max_in_features] * lin.pack_size
        for m, gid in zip(slots, member_ids):
            g, d = gen(lin.weight.device, _mix(seed, gid, j))
            b = inf[m] ** -0.5
            for p in (lin.weight, lin.bias):
                if p is None:
                    continue
                u = torch.rand(p.shape[1:], generator=g, device=d, dtype=p.dtype)
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


CheckpointKey = tuple[int, int]
"""(model id, the model's training step) of an evaluated checkpoint (`ModelCheckpointKey`,
`_training.py:531-540`)."""


class OnlineEnsemble:
    """The reference's `Ensemble` in online mode with an evaluation criterion
    (`_training.py:978-1183`), over checkpoint keys.

    After every epoch the candidates are the current members first, then the best
    checkpoints of finished members and the latest checkpoints of running members that are
    not members already (current members first: selection breaks ties by candidate order);
    greedy selection (`greedy_ensemble`, `ensemble.py:95-263`) picks from their validation
    predictions, and the rebuilt ensemble -- the mean of its members' predictions -- replaces
    the current one only when its score is higher.  A pool that holds exactly the current
    members counts as an update without improvement."""

    def __init__(self, score: PackScore, *, max_ensemble_size: int | None = 32, init_top_k: int = 1,
                 with_replacement: bool = False, early_stopping_patience: int | None = None) -> None:
        if early_stopping_patience is not None and early_stopping_patience < 0:
            raise ValueError('The early stopping patience must be non-negative')
        self.score = score
        self.max_ensemble_size = max_ensemble_size
        self.init_top_k = init_top_k
        self.with_replacement = with_replacement
        self.early_stopping_patience = early_stopping_patience
        self.member_keys: list[CheckpointKey] | None = None
        self.member_weights: Tensor | None = None
        self.best_score: float | None = None
        self.n_consecutive_bad_updates = 0

    def is_running(self) -> bool:
        return self.early_stopping_patience is None or self.n_consecutive_bad_updates <= self.early_stopping_patience

    def update(self, predictions: Callable[[CheckpointKey], Tensor], finished_best: list[CheckpointKey],
               running_latest: list[CheckpointKey]) -> bool:
        """`Ensemble.update` (`_training.py:1061-1183`); `predictions(key)` returns a
        checkpoint's validation predictions.  Returns whether the ensemble was replaced."""
        if not self.is_running():
            raise RuntimeError('the ensemble is finalized')
        candidates = list(finished_best) + list(running_latest)
        if not candidates or len(set(candidates)) != len(candidates):
            raise ValueError('candidate checkpoints must be non-empty and distinct')
        if self.member_keys is not None:
            current = set(self.member_keys)
            candidates = list(self.member_keys) + [k for k in candidates if k not in current]
            if set(candidates) == current:
                self.n_consecutive_bad_updates += 1
                return False
        pool = torch.stack([predictions(k) for k in candidates])
        idx, weights = greedy_ensemble(pool, score_fn=self.score, init_top_k=self.init_top_k,
                                       max_ensemble_size=self.max_ensemble_size,
                                       with_replacement=self.with_replacement)
        keys = [candidates[i] for i in idx.tolist()]
        if len(set(keys)) != len(keys):
            raise ValueError('The ensemble algorithm selected the same model checkpoint more than once')
        blend = compute_unsanitized_ensemble_predictions(pool[idx], weights)
        score = float(self.score(blend[None])[0])
        improved = not math.isnan(score) and (self.best_score is None or self.best_score < score)
        if improved:
            self.member_keys, self.member_weights, self.best_score = keys, weights, score
            self.n_consecutive_bad_updates = 0
        else:
            self.n_consecutive_bad_updates += 1
        return improved


@dataclasses.dataclass
class FitResult:
    """What `PackTrainer.fit` leaves behind (cf. `TrainedTabPack`, `_training.py:2021-2364`).
    Metrics are the validation criterion (lower is better for every loss here); checkpoint
    keys are (model id, model step)."""
    history: list[dict]            # per epoch: 'step' (training loop step), 'val_metric' and 'train_loss'
                                   # (n_models,) of the models trained that epoch (NaN for the others),
                                   # 'slot_model' (the model id each gathered slot trained, -1: none)
    best_step: Tensor              # (n_models,) model step of each model's best checkpoint
    best_metric: Tensor            # (n_models,) its validation metric
    ensemble_keys: list[CheckpointKey]
    ensemble_weights: Tensor | None
    ensemble_metric: float
    ensemble_history: list[dict]   # accepted updates: 'step', 'keys', 'metric'


class PackTrainer:
    """Trains a pack of TabPack MLPs, members sharded over the process group."""

    def __init__(self, *, n_members: int, model: dict, per_member_model: list[dict], optimizer: dict,
                 per_member_optimizer: list[dict] | None = None, loss: str, seed: int, device,
                 autocast_bf16: bool = True, group=None, cost: list[float] | None = None,
                 member_range: tuple[int, int] | None = None, init_on_host: bool = False,
                 n_models: int | None = None) -> None:
        """`member_range` pins this trainer to global members [lo, hi) without a process
        group (several shards on one device); otherwise the group's rank picks its range.
        `init_on_host` draws the initial parameters with host generators (the same values on
        every machine and device; slower for large packs).

        `n_models` (default `n_members`): models trained over the run through a pack of
        `n_members` slots.  `per_member_model` and `per_member_optimizer` then hold one entry
        per model id; slot s starts with model s, and `fit` gives the slots of finished
        models to the next ids.  The pack's maximum shapes (`model`) must fit every model."""
        if loss not in _LOSSES:
            raise ValueError(f'loss must be one of {_LOSSES}')
        self.n_models = n_members if n_models is None else int(n_models)
        if self.n_models < n_members:
            raise ValueError('n_models must be at least the number of pack slots')
        if len(per_member_model) != self.n_models or (per_member_optimizer is not None
                                                      and len(per_member_optimizer) != self.n_models):
            raise ValueError('one hyperparameter dict per model is required')
        if self.n_models > n_members and member_range is not None and tuple(member_range) != (0, n_members):
            raise ValueError('the replacement queue needs the whole pack: a process group or member_range '
                             '(0, n_members)')
        self.per_model = list(per_member_model)
        self.per_model_optimizer = None if per_member_optimizer is None else list(per_member_optimizer)
        self.slot_model = list(range(n_members))  # global slot -> model id it trains (-1: none)
        replacement = self.n_models > n_members
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
        # global ids of the rows that gather_members returns (this shard's alone with member_range)
        self.gathered_ids = list(range(n_members)) if member_range is None else list(range(lo, hi))
        self.loss = loss
        self.seed = int(seed)
        self.autocast = autocast_bf16
        self.device = torch.device(device)
        local = per_member_model[lo:hi]
        kw = _merge(model, _transpose(local))
        self.model = TabPack(pack_size=hi - lo, **kw).to(self.device)
        # this loop owns the gradients (the optimizer consumes them and sets them to None), so
        # each layer's weight gradient reuses the previous step's storage
        for mod in self.model.modules():
            if isinstance(mod, LinearPack):
                mod.reuse_weight_gradient = True
        # the backbone blocks' outputs feed only the next block (and the head), and their input
        # gradients only the previous block: a training step writes both into the previous
        # step's storage, whose padding is still zero
        for blk in self.model.backbone.blocks:
            blk.linear.reuse_activation_buffer = True
        self.model.output.reuse_activation_buffer = True
        self.model.backbone.set_member_base(lo)
        self.model.backbone._stream.seed = _mix(self.seed, 0xD0)  # one Philox key on every rank
        self._init_device = 'cpu' if init_on_host else None
        init_member_parameters_(self.model, seed=self.seed, member_ids=list(range(lo, hi)),
                                generator_device=self._init_device)
        okw = dict(optimizer)
        otype = okw.pop('type')
        if per_member_optimizer is not None:
            okw.update(_transpose(per_member_optimizer[lo:hi]))
        if otype == 'muon':
            groups = [MuonAdamWPack.make_muon_parameter_group(b.linear) for b in self.model.backbone.blocks]
            # the blocks a member's depth leaves out get an exactly zero gradient: the Muon step
            # does not read it (a key of this package's groups; the reference has no such key)
            for i, gr in enumerate(groups):
                if i > 0:
                    gr['muon_n_blocks'], gr['muon_block_index'] = self.model.backbone.n_blocks, i
                    # a gated member's momentum is zero as well: its gradient has always been
                    # zero, and `replace` zeroes the state of a member whose depth changes
                    gr['muon_gated_momentum_zero'] = True
            muon_params = {id(g['params'][0]) for g in groups}
            decay, no_decay = split_weight_decay(self.model)
            groups.append({'params': [p for p in no_decay if id(p) not in muon_params], 'weight_decay': 0.0})
            groups.append({'params': [p for p in decay if id(p) not in muon_params]})
            self.opt = MuonAdamWPack(groups, pack_size=hi - lo, allow_inplace_grad_mutation=False,
                                     support_replacement=replacement, **okw)
        elif otype == 'adamw':
            wd, nd = split_weight_decay(self.model)
            self.opt = AdamWPack([{'params': nd, 'weight_decay': 0.0}, {'params': wd}], pack_size=hi - lo,
                                 support_replacement=replacement, **okw)
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

    def fit_epoch(self, data: dict, *, batch_size: int, epoch: int,
                  on_step: Callable[[int, Tensor], None] | None = None) -> Tensor:
        """One epoch over `data` ({'x_num', 'x_cat', 'y'} on this device); returns the
        mean training loss of every member (P_total,) (gathered when sharded).  `on_step(i,
        losses)` sees each step's per-member losses of this rank (a device tensor)."""
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
            if on_step is not None:
                on_step(steps, losses.detach())
            steps += 1
        mean = total / max(steps, 1)
        return gather_members(mean, self.counts, self.group) if self.world > 1 else mean

    # ------------------------------------------------------------------ evaluation
    def _width_chunks(self, member_chunk: int) -> list[tuple[Tensor, int]]:
        """Member groups of `member_chunk` members in order of hidden width, each with its
        widest member's width (rounded up to 8): a group then runs with that maximum width
        instead of the pack's, so its activations are only as wide as its members need."""
        P = self.hi - self.lo
        outf = self.model.backbone.blocks[0].linear.out_features
        widths = outf.tolist() if outf is not None else [self.model.backbone.blocks[0].linear.max_out_features] * P
        order = sorted(range(P), key=lambda m: (widths[m], m))
        chunks = []
        for c in range(0, P, member_chunk):
            members = order[c: c + member_chunk]
            mw = -(-max(widths[m] for m in members) // 8) * 8
            chunks.append((torch.tensor(members, device=self.device), mw))
        return chunks

    @torch.no_grad()
    def predict_local(self, data: dict, *, eval_batch_size: int = 32768, member_chunk: int | None = None) -> Tensor:
        """Transformed predictions of this rank's members on a shared dataset.  `member_chunk`
        runs the members in groups of that size (bounds the activations of wide packs on large
        batches: each group is a `pack_idx` selection of the pack, of members of similar width
        that run with their own maximum width)."""
        self.model.eval()
        n = len(data['y']) if 'y' in data else len(next(iter(data.values())))
        P = self.hi - self.lo
        chunks = None if member_chunk is None or member_chunk >= P else self._width_chunks(member_chunk)
        parts = []
        for i in range(0, n, eval_batch_size):
            xn = data['x_num'][i: i + eval_batch_size] if 'x_num' in data else None
            xc = data['x_cat'][i: i + eval_batch_size] if 'x_cat' in data else None
            if chunks is None:
                with torch.autocast('cuda', dtype=torch.bfloat16, enabled=self.autocast):
                    out = self.model(xn, xc)
                parts.append(transform(self.loss, out.float()))
                continue
            full = None
            for idx, mw in chunks:
                with torch.autocast('cuda', dtype=torch.bfloat16, enabled=self.autocast):
                    out = self.model(xn, xc, idx, max_width=mw)
                out = transform(self.loss, out.float())
                if full is None:
                    full = out.new_empty((P, *out.shape[1:]))
                full.index_copy_(0, idx, out)
            parts.append(full)
        return torch.cat(parts, 1)

    def _score(self, y_val: Tensor) -> PackScore:
        return PackScore({'mse': 'mse', 'bce': 'bce', 'ce': 'ce'}[self.loss], y_val, maximize=False)

    def predict(self, data: dict, *, eval_batch_size: int = 32768) -> Tensor:
        """Transformed predictions of every member (gathered over ranks when sharded)."""
        local = self.predict_local(data, eval_batch_size=eval_batch_size)
        return gather_members(local, self.counts, self.group) if self.world > 1 else local

    def _freeze(self, local_idx: list[int]) -> None:
        """Stop updating these members: a zero learning rate makes every optimizer update of
        theirs (weight decay included, p * (1 - lr * wd)) leave the parameters unchanged."""
        if not local_idx:
            return
        idx = torch.tensor(local_idx, device=self.device)
        P = self.hi - self.lo
        for g in self.opt.param_groups:
            for key in ('lr', 'adamw_lr', 'muon_lr'):
                if key not in g:
                    continue
                v = g[key]
                if not isinstance(v, Tensor):
                    v = torch.full((P,), float(v), device=self.device)
                v = v.to(self.device, torch.float32).clone()
                v[idx] = 0.0
                g[key] = v

    def _replace_local(self, pairs: list[tuple[int, int]]) -> None:
        """`pack_replace` (`_training.py:860-924`) on this rank's slots: (local slot, model id)
        pairs take the models' shapes and hyperparameters, fresh optimizer state (the Muon
        update scales follow the new shapes) and parameters initialised from the model ids."""
        if not pairs:
            return
        slots = [sl for sl, _ in pairs]
        models = [m for _, m in pairs]
        idx = torch.tensor(slots, device=self.device)
        self.model.replace(pack_idx=idx, **_transpose([self.per_model[m] for m in models]))
        okw = {} if self.per_model_optimizer is None else _transpose([self.per_model_optimizer[m] for m in models])
        if isinstance(self.opt, MuonAdamWPack):
            self.opt.replace(pack_idx=idx, module=self.model, **okw)
        else:
            self.opt.replace(pack_idx=idx, **okw)
        init_member_parameters_(self.model, seed=self.seed, member_ids=models, pack_idx=slots,
                                generator_device=self._init_device)

    def fit(self, train: dict, val: dict, *, batch_size: int, max_epochs: int | list[int],
            early_stopping_patience: int | None = None, ensemble: OnlineEnsemble | None = None,
            eval_batch_size: int = 32768) -> FitResult:
        """The reference's training loop (`_training.py:2643-2960`): train an epoch, evaluate
        every slot's model on `val`, update each model's best checkpoint
        (`update_training_state`, `_training.py:754-821`; a model's first evaluation is its
        first best checkpoint even when NaN), stop the models that reached their `max_epochs`
        (one value, or one per model id) or ran out of patience (their best checkpoints are then
        final), update `ensemble` (by default an `OnlineEnsemble` over the validation criterion,
        at most 32 members), then give the freed slots to the next model ids while any are left
        (`shard.assign_replacements`).  Ends when every model has finished."""
        M = self.n_models
        max_ep = [max_epochs] * M if isinstance(max_epochs, int) else list(max_epochs)
        if len(max_ep) != M or any(int(v) <= 0 for v in max_ep):
            raise ValueError('max_epochs must be positive (one value, or one per model)')
        score = self._score(val['y'])
        if ensemble is None:
            ensemble = OnlineEnsemble(score)
        ids = self.gathered_ids                   # global slots whose predictions predict() returns
        S = len(ids)
        occ = [self.slot_model[g] for g in ids]   # model id each slot trains (-1: none)
        steps_per_epoch = math.ceil(len(train['y']) / batch_size)
        max_steps = [int(v) * steps_per_epoch for v in max_ep]
        steps, n_bad, best_step = [0] * M, [0] * M, [0] * M
        best_metric = [math.nan] * M
        active = [m >= 0 for m in occ]
        fresh = list(active)                      # the slot's model has not been evaluated yet
        next_model = 1 + max(self.slot_model)
        best_pred: Tensor | None = None           # (S, ...) best predictions of each slot's model
        finished: list[CheckpointKey] = []
        store: dict[CheckpointKey, Tensor] = {}
        history: list[dict] = []
        ensemble_history: list[dict] = []
        loop_step = 0
        epoch = 0
        while any(active):
            loss = self.fit_epoch(train, batch_size=batch_size, epoch=epoch)
            epoch += 1
            loop_step += steps_per_epoch
            for i in range(S):
                if active[i]:
                    steps[occ[i]] += steps_per_epoch
            preds = self.predict(val, eval_batch_size=eval_batch_size)
            latest = (-score(preds)).double().cpu().tolist()
            if best_pred is None:
                best_pred = preds.clone()
            rows = []
            for i in range(S):
                if not active[i]:
                    continue
                m, x = occ[i], latest[i]
                improved = not math.isnan(x) and (fresh[i] or math.isnan(best_metric[m]) or x < best_metric[m])
                n_bad[m] = 0 if improved else n_bad[m] + 1
                if improved or fresh[i]:
                    best_metric[m], best_step[m] = x, steps[m]
                    rows.append(i)
                fresh[i] = False
            if rows:
                r = torch.tensor(rows, device=preds.device)
                best_pred[r] = preds[r]
            running = [active[i] and steps[occ[i]] < max_steps[occ[i]]
                       and (early_stopping_patience is None or n_bad[occ[i]] <= early_stopping_patience)
                       for i in range(S)]
            stopped = [i for i in range(S) if active[i] and not running[i]]
            finished += [(occ[i], best_step[occ[i]]) for i in stopped]
            running_latest = [(occ[i], steps[occ[i]]) for i in range(S) if running[i]]
            slot_of = {occ[i]: i for i in range(S) if active[i]}

            def lookup(key: CheckpointKey) -> Tensor:
                i = slot_of.get(key[0])
                if i is not None and key[1] == steps[key[0]]:
                    return preds[i]
                if i is not None and key[1] == best_step[key[0]]:
                    return best_pred[i]
                return store[key]

            if ensemble.is_running() and (finished or running_latest):
                if ensemble.update(lookup, finished, running_latest):
                    ensemble_history.append({'step': loop_step, 'keys': list(ensemble.member_keys),
                                             'metric': -ensemble.best_score})
            # keep the predictions that later updates may need: finished models' best
            # checkpoints and the current ensemble members (`rebuild_checkpoint_store`)
            required = set(finished) | set(ensemble.member_keys or [])
            store = {k: (store[k] if k in store else lookup(k).clone()) for k in required}
            vm = [math.nan] * M
            tl = torch.full((M,), math.nan, dtype=loss.dtype)
            loss_h = loss.cpu()
            for i in range(S):
                if active[i]:
                    vm[occ[i]] = latest[i]
                    tl[occ[i]] = loss_h[i]
            history.append({'step': loop_step, 'val_metric': torch.tensor(vm, dtype=torch.float64),
                            'train_loss': tl, 'slot_model': list(occ)})
            # the replacement queue: freed slots take the next model ids, the rest stop training
            pending = M - len(finished) - sum(running)
            pairs = assign_replacements([ids[i] for i in stopped], next_model_id=next_model, n_pending=pending)
            next_model += len(pairs)
            refilled = {g for g, _ in pairs}
            self._freeze([ids[i] - self.lo for i in stopped
                          if ids[i] not in refilled and self.lo <= ids[i] < self.hi])
            self._replace_local([(g - self.lo, m) for g, m in pairs if self.lo <= g < self.hi])
            pos = {g: i for i, g in enumerate(ids)}
            for i in stopped:
                occ[i] = -1
                self.slot_model[ids[i]] = -1
            for g, m in pairs:
                self.slot_model[g] = m
                if g in pos:
                    occ[pos[g]] = m
                    fresh[pos[g]] = True
            was_stopped = set(stopped)
            active = [running[i] or (occ[i] >= 0 and i in was_stopped) for i in range(S)]
        return FitResult(history=history, best_step=torch.tensor(best_step),
                         best_metric=torch.tensor(best_metric, dtype=torch.float64),
                         ensemble_keys=list(ensemble.member_keys or []), ensemble_weights=ensemble.member_weights,
                         ensemble_metric=math.nan if ensemble.best_score is None else -ensemble.best_score,
                         ensemble_history=ensemble_history)

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


__all__ = ['PackTrainer', 'PackPredictor', 'EpochResult', 'FitResult', 'OnlineEnsemble', 'CheckpointKey',
           'init_member_parameters_', 'member_loss', 'transform', 'assert_finite']
