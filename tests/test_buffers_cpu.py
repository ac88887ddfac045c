"""Host-side rules of the storage that a trainer's layers reuse from step to step (no GPU):
a buffer is handed out again only when nothing else holds its storage and its key (widths
and depths) is unchanged; otherwise a zeroed new one replaces it."""

import torch

from tabpack_b200.nn import _activation_buffer, _weight_gradient_buffer


def test_activation_buffer_reused_only_when_released():
    slot = {}
    a = _activation_buffer(slot, (2, 3, 8), torch.float32, torch.device('cpu'), key='k')
    assert a is not None and torch.count_nonzero(a) == 0
    a.fill_(5.0)
    ptr = a.data_ptr()
    # still held (a pending backward would read it): a new, zeroed buffer
    b = _activation_buffer(slot, (2, 3, 8), torch.float32, torch.device('cpu'), key='k')
    assert b.data_ptr() != ptr and torch.count_nonzero(b) == 0
    del a
    ptr_b = b.data_ptr()
    del b
    # released: the same storage again, contents kept (the kernels rely on its zero padding)
    c = _activation_buffer(slot, (2, 3, 8), torch.float32, torch.device('cpu'), key='k')
    assert c.data_ptr() == ptr_b
    del c
    # a view that outlives its base still holds the storage
    d = _activation_buffer(slot, (2, 3, 8), torch.float32, torch.device('cpu'), key='k')
    view = d[0]
    del d
    e = _activation_buffer(slot, (2, 3, 8), torch.float32, torch.device('cpu'), key='k')
    assert e.data_ptr() != view.data_ptr()
    del view, e


def test_activation_buffer_rebuilt_on_new_key_or_shape():
    slot = {}
    a = _activation_buffer(slot, (2, 4), torch.float32, torch.device('cpu'), key=('w', 1))
    a.fill_(1.0)
    del a
    b = _activation_buffer(slot, (2, 4), torch.float32, torch.device('cpu'), key=('w', 2))
    assert torch.count_nonzero(b) == 0  # widths changed: padding must be rebuilt as zeros
    del b
    c = _activation_buffer(slot, (3, 4), torch.float32, torch.device('cpu'), key=('w', 2))
    assert c.shape == (3, 4) and torch.count_nonzero(c) == 0
    d = _activation_buffer(slot, (3, 4), torch.bfloat16, torch.device('cpu'), key=('w', 2))
    assert d.dtype == torch.bfloat16


def test_weight_gradient_buffer_reused_after_the_gradient_is_dropped():
    import weakref

    slot = {}
    g = _weight_gradient_buffer(slot, (2, 4, 4), torch.device('cpu'), key='k')
    assert torch.count_nonzero(g) == 0
    slot['ref'] = weakref.ref(g)
    ptr = g.data_ptr()
    h = _weight_gradient_buffer(slot, (2, 4, 4), torch.device('cpu'), key='k')
    assert h.data_ptr() != ptr  # the previous gradient is still alive
    slot['ref'] = weakref.ref(h)
    ptr_h = h.data_ptr()
    del g, h
    i = _weight_gradient_buffer(slot, (2, 4, 4), torch.device('cpu'), key='k')
    assert i.data_ptr() == ptr_h


def test_prediction_groups_follow_width_order():
    """`PackTrainer.predict_local` groups members of similar width; each group's maximum width
    is its widest member's, rounded up to 8, and every member appears once."""
    from types import SimpleNamespace

    from tabpack_b200.training import PackTrainer

    widths = [640, 128, 1024, 256, 250, 136, 900]
    lin = SimpleNamespace(out_features=torch.tensor(widths), max_out_features=1024)
    fake = SimpleNamespace(lo=0, hi=len(widths), device='cpu',
                           model=SimpleNamespace(backbone=SimpleNamespace(blocks=[SimpleNamespace(linear=lin)])))
    chunks = PackTrainer._width_chunks(fake, 3)
    members = [m for idx, _ in chunks for m in idx.tolist()]
    assert sorted(members) == list(range(len(widths)))
    assert [idx.tolist() for idx, _ in chunks] == [[1, 5, 4], [3, 0, 6], [2]]
    assert [mw for _, mw in chunks] == [256, 904, 1024]
