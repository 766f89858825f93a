"""Lazy-fusion capture toggles (mirrors src/rushlite/capture_mode.py of the
reference): ops on CUDA Variables inside the block are recorded and fused on
first use of their result."""
from contextlib import contextmanager
from functools import wraps

from ._C import is_capture_enabled, set_capture_enabled


@contextmanager
def capture_on(enable: bool = True):
    prev = is_capture_enabled()
    try:
        set_capture_enabled(enable)
        yield
    finally:
        set_capture_enabled(prev)


def capture(enable: bool = True):
    def decorator(fn):
        @wraps(fn)
        def _wrapper(*args, **kwargs):
            with capture_on(enable):
                return fn(*args, **kwargs)

        return _wrapper

    return decorator
