"""Switching the reference's scan module over to the B200 kernels, by device.

The reference keeps its scan entry points in ``models/selective_scan.py``
(``selective_scan_fast`` :246, ``selective_scan_ref`` :34, ``parallel_scan`` :66,
``sequential_scan`` :91).  A maintainer adds two lines at the END of that file:

    from swiftx_b200.integrate import patch_reference_module
    patch_reference_module(globals())

Each of the four names is then replaced by a function with the same signature that
sends CUDA tensors to ``swiftx_b200`` (the sm_100a kernels) and passes anything else to
the reference's own function, which it keeps unchanged.  The reference's CPU code paths
(its CPU test suite, CPU training) therefore keep running the reference's own code,
while SiftBlock / SiftLM on a B200 pick the kernels up without any other change.  The
module's internal callers (``_scan`` calls ``parallel_scan``) see the patched names
too, so they dispatch the same way.

Nothing here computes on the CPU: for non-CUDA tensors the functions call back into
the reference module's originals, and the kernel library is loaded (and fails loudly if
it was not built) the first time a CUDA tensor arrives.
"""
import functools

from . import selective_scan as _swx

_NAMES = ("selective_scan_fast", "selective_scan_ref", "parallel_scan", "sequential_scan")


def _on_cuda(x):
    return getattr(x, "is_cuda", False)


def _dispatch(name, original):
    ours = getattr(_swx, name)

    @functools.wraps(original)
    def fn(*args, **kwargs):
        first = args[0] if args else next(iter(kwargs.values()), None)
        if _on_cuda(first):
            return ours(*args, **kwargs)
        return original(*args, **kwargs)

    fn.__swiftx_original__ = original
    return fn


def patch_reference_module(namespace):
    """Replace the reference scan entry points found in ``namespace`` (the module's
    ``globals()``) by device-dispatching versions.  Idempotent; returns the patched names."""
    done = []
    for name in _NAMES:
        orig = namespace.get(name)
        if orig is None:
            continue
        orig = getattr(orig, "__swiftx_original__", orig)
        namespace[name] = _dispatch(name, orig)
        done.append(name)
    return done
