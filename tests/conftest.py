import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, 'tests', 'golden')


def pytest_configure(config):
    config.addinivalue_line('markers', 'gpu: needs a B200 (sm_100a) and the built CUDA library')


@pytest.fixture
def golden():
    import numpy as np

    def load(name):
        return np.load(os.path.join(GOLDEN, name))

    return load


@pytest.fixture
def reference():
    """The reference package `tabpackage`, imported from TABPACK_REFERENCE_SRC (its `src`
    directory) or the path; tests that need it are skipped where it is not available."""
    src = os.environ.get('TABPACK_REFERENCE_SRC')
    if src and src not in sys.path:
        sys.path.insert(0, src)
    try:
        import tabpackage
        import tabpackage._training  # noqa: F401
        import tabpackage.nn  # noqa: F401
        import tabpackage.optim  # noqa: F401
    except ImportError:
        pytest.skip('the reference package `tabpackage` is not importable (set TABPACK_REFERENCE_SRC)')
    return tabpackage


def pytest_sessionstart(session):
    # The CUDA library is built in-tree; rebuild it when a source is newer.
    from tabpack_b200.csrc import build

    build.build()
