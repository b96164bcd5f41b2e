"""ctypes binding of libsumac_b200.so (the C ABI declared in include/sumac_b200.h).

The library is built in-tree by ``sumac_b200.build``. Loading fails loudly when it is missing:
there is no CPU or library fallback for any operation of this package.
"""
from __future__ import annotations

import ctypes as C
import os
import threading

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_lib", "libsumac_b200.so")

SUMAC_TF32 = 1
SUMAC_3XTF32 = 3

_lock = threading.Lock()
_lib = None

p = C.c_void_p
i64 = C.c_int64
i32 = C.c_int
f32 = C.c_float
sz = C.c_size_t
u64 = C.c_ulonglong

_SIGS = {
    "sumac_version": (i32, []),
    "sumac_num_sms": (i32, [i32]),
    "sumac_padded_rank": (i32, [i32]),
    "sumac_last_error": (C.c_char_p, []),
    "sumac_set_timeout_ns": (None, [u64]),
    "sumac_kernel_launches": (C.c_longlong, []),
    "sumac_gather_owned_rows": (i32, [p, i64, i64, p, i64, i32, p, p]),
    "sumac_relu_product_splits": (i32, [i64, i64, i32, i32]),
    "sumac_relu_product": (i32, [p, i64, p, p, p, p, i64, i64, i32, i32, p, p, p]),
    "sumac_relu_bat_c_workspace_bytes": (sz, [i64, i64, i32, i32]),
    "sumac_relu_bat_c": (i32, [p, p, p, i64, i64, i32, p, i32, p, sz, p, p]),
    "sumac_relu_bat_c_mode": (i32, [p, p, p, i64, i64, i32, p, i32, i32, p, sz, p, p]),
    "sumac_relu_bat_reduce_workspace_bytes": (sz, [i64, i64, i32, i32]),
    "sumac_relu_bat_reduce": (i32, [p, p, i64, i64, i32, p, i32, p, sz, p, p]),
    "sumac_noalloc_scratch_bytes": (sz, []),
    "sumac_relu_bat_reduce_noalloc": (i32, [p, p, i64, i64, i32, p, i32, p, p]),
    "sumac_masked_product_workspace_bytes": (sz, [i64, i64, i32, i32]),
    "sumac_masked_product": (i32, [p, p, p, i64, i64, i32, p, p, p, i32, p, sz, p, p]),
    "sumac_salsa_update_workspace_bytes": (sz, [i64, i64, i32, i32]),
    "sumac_salsa_block_update": (i32, [p, i64, p, i64, p, p, i64, i32, p, p, f32, f32, p, i32,
                                       p, sz, p, p]),
    "sumac_block_csr_workspace_bytes": (sz, [i64, i64, i32, i64]),
    "sumac_block_csr_build": (i32, [p, i64, i32, p, p, p, i64, i64, p, p, p, sz, p]),
    "sumac_gd_grad_workspace_bytes": (sz, [i64, i64, i32, i32]),
    "sumac_gd_block_grad": (i32, [p, p, i64, i32, p, i64, p, p, p, p, p, p, i32, i32, p, sz,
                                  p, p]),
    "sumac_eval_terms_workspace_bytes": (sz, [i64, i64, i64, i32, i32]),
    "sumac_eval_terms": (i32, [p, p, i64, i64, i32, p, p, p, i64, p, i32, p, sz, p, p]),
    "sumac_eval_terms_fnnz": (i32, [p, p, i64, i64, i32, p, p, p, i64, p, i32, p, sz, p, p]),
    "sumac_block_loss_workspace_bytes": (sz, [i64, i64, i32, i32]),
    "sumac_block_loss_terms": (i32, [p, p, i64, i32, p, i64, p, p, p, i32, i32, p, sz, p, p]),
    "sumac_adam_step": (i32, [p, p, p, p, i64, f32, f32, f32, f32, f32, p]),
    "sumac_grad_sumsq": (i32, [p, i64, p, p]),
    "sumac_sgd_step": (i32, [p, p, p, i64, f32, f32, i32, p, f32, p]),
    "sumac_fill_zero": (i32, [p, i64, p]),
    "sumac_assemble_rows_p2p": (i32, [p, i64, i64, p, i64, i32, i64, p, p, p, i32, i32, p, p]),
    "sumac_init_factor": (i32, [p, p, p, i64, p, i32, f32, p, p]),
    "sumac_init_scale_workspace_bytes": (sz, []),
    "sumac_init_scale_terms": (i32, [p, p, i32, p, p, p, i64, p, p, sz, p]),
    "sumac_wait_flag": (i32, [p, p, u64, p]),
}


def exported_symbols():
    """Names of every entry point this binding declares (all must be exported by the library)."""
    return list(_SIGS)


def lib():
    """Load (once) and return the shared library with typed signatures."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"sumac_b200: native library not found at {LIB_PATH}; build it with "
                    "`python -m sumac_b200.build` (there is no fallback implementation)")
            L = C.CDLL(LIB_PATH)
            for name, (res, args) in _SIGS.items():
                fn = getattr(L, name)
                fn.restype = res
                fn.argtypes = args
            _lib = L
    return _lib


class NativeError(RuntimeError):
    pass


def check(rc: int, what: str) -> None:
    if rc != 0:
        msg = lib().sumac_last_error().decode(errors="replace")
        if rc == -1:
            raise ValueError(f"{what}: {msg}")
        if rc == -2:
            raise NotImplementedError(f"{what}: {msg}")
        raise NativeError(f"{what}: {msg} (status {rc})")


def ptr(t) -> int | None:
    if t is None:
        return None
    return t.data_ptr()


def stream_ptr(device=None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


# ------------------------------------------------------------------ per-device state
_err_words: dict[int, torch.Tensor] = {}
_workspaces: dict[tuple[int, str], torch.Tensor] = {}


def err_word(device) -> torch.Tensor:
    """Per-device int32 word where kernels report timeouts / singular solves."""
    idx = torch.device(device).index or 0
    w = _err_words.get(idx)
    if w is None:
        w = torch.zeros(1, dtype=torch.int32, device=f"cuda:{idx}")
        _err_words[idx] = w
    return w


DEVICE_ERRORS = {
    1: "a TMA stage never arrived (timeout)",
    2: "a pipeline stage was never released (timeout)",
    3: "an MMA result never arrived (timeout)",
    4: "the epilogue never released a TMEM buffer (timeout)",
    5: "the output accumulator wait timed out",
    6: "the row-tile load wait timed out",
    7: "flag wait timed out",
    8: "a peer GPU did not signal the row exchange in time",
    100: "singular Gram matrix in the SALSA least-squares solve",
}


def read_device_error(device, reset: bool = True) -> int:
    """Synchronises with the device and returns (and optionally clears) its error word."""
    w = err_word(device)
    code = int(w.item())
    if reset and code:
        w.zero_()
    return code


def raise_device_error(device) -> None:
    """Raise on a device-side timeout. An exactly singular Gram matrix (code 100) only warns: the
    reference's solver also carries on with whatever the solve returns."""
    code = read_device_error(device)
    if code == 100:
        import warnings
        warnings.warn("sumac_b200: singular Gram matrix in a SALSA block solve")
        return
    if code:
        raise NativeError(f"sumac_b200 device error {code}: {DEVICE_ERRORS.get(code, 'unknown')}")


def workspace(device, nbytes: int, tag: str = "main") -> torch.Tensor:
    """A grow-only device byte buffer per (device, tag), allocated through torch's allocator."""
    idx = torch.device(device).index or 0
    key = (idx, tag)
    w = _workspaces.get(key)
    if w is None or w.numel() < nbytes:
        w = torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=f"cuda:{idx}")
        _workspaces[key] = w
    return w
