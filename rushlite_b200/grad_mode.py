"""no_grad (mirrors src/rushlite/grad_mode.py of the reference): ops inside
the block record no backward function."""
from contextlib import contextmanager

from ._C import is_grad_enabled, set_grad_enabled


@contextmanager
def no_grad():
    prev = is_grad_enabled()
    try:
        set_grad_enabled(False)
        yield
    finally:
        set_grad_enabled(prev)
