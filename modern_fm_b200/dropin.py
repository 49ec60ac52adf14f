"""Install this engine beneath the reference's unchanged Python package.

The reference's `python/modern_fm/_backend.py` imports `modern_fm._rust`
(_backend.py:19-22) and routes both its CPU calls (use_cuda=False,
*_predict_fast_*, *_predict_{csr,dense}) and its CUDA calls (use_cuda=True,
*_predict_cuda_csr, has_cuda) through that one module. `make_rust_module`
builds a module with every name the reference's PyO3 module registers
(rust/src/lib.rs:1592-1614): the CUDA names come from this engine
(`modern_fm_b200._rust`), the CPU names from `cpu_backend` — normally the
reference's own compiled `_rust` extension, whose CPU engine stays the CPU
engine. `install` puts that module in place as `modern_fm._rust`.

    import modern_fm_b200.dropin as d
    d.install(cpu_backend=reference_rust_module)
    from modern_fm import FMClassifier
    FMClassifier(backend="cuda").fit(X, y)   # trains on the B200 engine
"""

from __future__ import annotations

import sys
import types

from . import _rust as engine

CPU_ONLY = ("fm_predict_fast_dense", "fm_predict_fast_csr", "ffm_predict_dense",
            "ffm_predict_csr", "fwfm_predict_dense", "fwfm_predict_csr")
FIT = ("fm_fit_csr", "fm_fit_multiclass_csr", "ffm_fit_csr", "ffm_fit_multiclass_csr",
       "fwfm_fit_csr", "fwfm_fit_multiclass_csr")
CUDA_ONLY = ("has_cuda", "fm_predict_cuda_csr", "ffm_predict_cuda_csr", "fwfm_predict_cuda_csr")


def _fit_router(name, cpu_fn):
    cuda_fn = getattr(engine, name)

    def fit(*args, use_cuda=False, **kwargs):
        if use_cuda:
            return cuda_fn(*args, use_cuda=True, **kwargs)
        if cpu_fn is None:
            raise ValueError(f"{name}(use_cuda=False) needs a CPU backend; none was installed")
        return cpu_fn(*args, use_cuda=False, **kwargs)

    fit.__name__ = name
    fit.__doc__ = f"{name}: use_cuda=True -> B200 engine, otherwise the CPU backend."
    return fit


def make_rust_module(cpu_backend=None, name="modern_fm._rust") -> types.ModuleType:
    """A module exposing the reference `_rust` surface (see module docstring)."""
    mod = types.ModuleType(name)
    mod.__doc__ = "modern_fm._rust composed from the B200 engine and a CPU backend"
    for n in CUDA_ONLY:
        setattr(mod, n, getattr(engine, n))
    for n in CPU_ONLY:
        fn = getattr(cpu_backend, n, None) if cpu_backend is not None else None
        if fn is not None:
            setattr(mod, n, fn)
    for n in FIT:
        setattr(mod, n, _fit_router(n, getattr(cpu_backend, n, None) if cpu_backend else None))
    return mod


def install(cpu_backend=None, package="modern_fm") -> types.ModuleType:
    """Register the composed module as `<package>._rust`; if the package's
    `_backend` is already imported, point it at the new module too."""
    mod = make_rust_module(cpu_backend, name=f"{package}._rust")
    sys.modules[f"{package}._rust"] = mod
    pkg = sys.modules.get(package)
    if pkg is not None:
        setattr(pkg, "_rust", mod)
    backend = sys.modules.get(f"{package}._backend")
    if backend is not None:
        backend._rust = mod
    return mod
