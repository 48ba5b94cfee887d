"""ctypes binding of libaestrix_cuda (the C ABI declared in include/aestrix_cuda.h).

The shared library is built in-tree by ``make -C aestrix_b200/csrc`` (or
``__graft_entry__.build()``) and loaded from this package directory. There is
no fallback: if the library is missing or fails to load, :func:`lib` raises.
"""
from __future__ import annotations

import ctypes as C
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libaestrix_cuda.so")

AEX_OK = 0
AEX_ERR_INVALID_ARG = 1
AEX_ERR_UNSUPPORTED = 2
AEX_ERR_CUDA = 3
AEX_ERR_NCCL = 4
AEX_ERR_TIMEOUT = 5
AEX_ERR_OOM = 6
AEX_ERR_DEVICE = 7

AEX_DTYPE_BF16 = 0
AEX_DTYPE_F32 = 1

_ERR_NAMES = {
    AEX_ERR_INVALID_ARG: "AEX_ERR_INVALID_ARG",
    AEX_ERR_UNSUPPORTED: "AEX_ERR_UNSUPPORTED",
    AEX_ERR_CUDA: "AEX_ERR_CUDA",
    AEX_ERR_NCCL: "AEX_ERR_NCCL",
    AEX_ERR_TIMEOUT: "AEX_ERR_TIMEOUT",
    AEX_ERR_OOM: "AEX_ERR_OOM",
    AEX_ERR_DEVICE: "AEX_ERR_DEVICE",
}


class AexError(RuntimeError):
    """Non-zero status from a libaestrix_cuda entry point."""

    def __init__(self, code: int, message: str):
        super().__init__(f"{_ERR_NAMES.get(code, code)}: {message}")
        self.code = code


class aex_bshd(C.Structure):
    _fields_ = [
        ("data", C.c_void_p),
        ("stride_b", C.c_int64),
        ("stride_s", C.c_int64),
        ("stride_h", C.c_int64),
    ]


class aex_attention_args(C.Structure):
    _fields_ = [
        ("q", aex_bshd),
        ("k", aex_bshd),
        ("v", aex_bshd),
        ("out", aex_bshd),
        ("batch", C.c_int),
        ("seq", C.c_int),
        ("heads", C.c_int),
        ("head_dim", C.c_int),
        ("norm_q_weight", C.c_void_p),
        ("norm_k_weight", C.c_void_p),
        ("eps", C.c_float),
        ("rope_cos", C.c_void_p),
        ("rope_sin", C.c_void_p),
        ("scale", C.c_float),
    ]


class aex_sp_op(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("kind", "send_to", "recv_from", "slot", "part", "wait_exchange", "stream")]


AEX_SP_OP_EXCHANGE, AEX_SP_OP_ATTEND, AEX_SP_OP_MERGE = 0, 1, 2


def sp_plan(world: int, rank: int) -> list[aex_sp_op]:
    """The overlap schedule's steps for `rank` (aex_sp_plan)."""
    n = lib().aex_sp_plan(world, rank, None, 0)
    if n < 0:
        raise ValueError(f"no overlap plan for world {world} rank {rank}")
    ops = (aex_sp_op * n)()
    if lib().aex_sp_plan(world, rank, ops, n) != n:
        raise RuntimeError("aex_sp_plan")
    return list(ops)


class aex_dit_config(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("hidden", "heads", "n_double", "n_single", "mlp_hidden", "in_channels",
                                       "text_dim", "timestep_dim", "l_txt", "l_img")] + [
        ("rms_eps", C.c_float), ("ln_eps", C.c_float)]


# (name, restype, argtypes) for every symbol declared in include/aestrix_cuda.h.
_VP = C.c_void_p
_SIGNATURES = [
    ("aex_abi_version", C.c_int, []),
    ("aex_ctx_create", C.c_int, [C.c_int, C.POINTER(_VP)]),
    ("aex_ctx_destroy", None, [_VP]),
    ("aex_last_error_string", C.c_char_p, [_VP]),
    ("aex_sync", C.c_int, [_VP, _VP, C.c_int]),
    ("aex_device_status", C.c_int, [_VP, C.POINTER(C.c_int)]),
    ("aex_device_sm_count", C.c_int, [_VP]),
    ("aex_joint_attention", C.c_int, [_VP, C.POINTER(aex_attention_args), _VP]),
    ("aex_joint_attention_scratch_bytes", C.c_size_t, [C.POINTER(aex_attention_args)]),
    ("aex_joint_attention_ws", C.c_int, [_VP, C.POINTER(aex_attention_args), _VP, C.c_size_t, _VP]),
    ("aex_joint_attention_noalloc", C.c_int, [_VP, C.POINTER(aex_attention_args), _VP]),
    ("aex_rope_tables", C.c_int, [_VP, _VP, C.c_int, C.c_float, _VP, C.c_int, _VP, _VP, _VP]),
    ("aex_dequantize_mlx", C.c_int, [_VP, _VP, _VP, _VP, C.c_int, C.c_int, C.c_int, C.c_int, _VP, _VP]),
    ("aex_qweight_create", C.c_int,
     [_VP, _VP, _VP, _VP, C.c_int, C.c_int, C.c_int, C.c_int, C.POINTER(_VP), _VP]),
    ("aex_qweight_destroy", None, [_VP]),
    ("aex_qweight_shape", C.c_int, [_VP, C.POINTER(C.c_int), C.POINTER(C.c_int)]),
    ("aex_qweight_dequantize", C.c_int, [_VP, _VP, _VP, _VP]),
    ("aex_qmm", C.c_int, [_VP, _VP, _VP, C.c_int64, C.c_int, _VP, C.c_int64, C.c_int, _VP]),
    ("aex_qmm_ex", C.c_int, [_VP, _VP, _VP, C.c_int, C.c_int64, C.c_int, _VP, C.c_int64, C.c_int, _VP]),
    ("aex_dit_create", C.c_int, [_VP, C.POINTER(aex_dit_config), C.POINTER(_VP)]),
    ("aex_dit_destroy", None, [_VP]),
    ("aex_dit_load_linear", C.c_int, [_VP, C.c_char_p, _VP, _VP, _VP, C.c_int, C.c_int, _VP]),
    ("aex_dit_load_norm", C.c_int, [_VP, C.c_char_p, _VP, _VP]),
    ("aex_dit_set_rope", C.c_int, [_VP, _VP, _VP, _VP]),
    ("aex_dit_project_context", C.c_int, [_VP, _VP, _VP]),
    ("aex_dit_set_timestep", C.c_int, [_VP, C.c_float, _VP]),
    ("aex_dit_forward", C.c_int, [_VP, _VP, _VP, _VP]),
    ("aex_dit_denoise_step", C.c_int, [_VP, _VP, _VP, C.c_float, _VP]),
    ("aex_dit_denoise", C.c_int, [_VP, _VP, C.c_int, _VP]),
    ("aex_dit_load_safetensors", C.c_int, [_VP, C.c_char_p, _VP, _VP, _VP]),
    ("aex_dit_set_sequence_parallel", C.c_int, [_VP, _VP, C.c_int, C.c_int]),
    ("aex_safetensors_scan", C.c_int, [C.c_char_p, C.c_char_p, C.c_size_t]),
    ("aex_comm_unique_id", C.c_int, [_VP]),
    ("aex_comm_create", C.c_int, [_VP, C.c_int, C.c_int, _VP, C.c_int, C.POINTER(_VP)]),
    ("aex_comm_destroy", None, [_VP]),
    ("aex_comm_abort", C.c_int, [_VP]),
    ("aex_ring_attention", C.c_int, [_VP, _VP, C.POINTER(aex_attention_args), _VP]),
    ("aex_sp_schedule", C.c_int, [C.c_int, C.c_int, C.c_int]),
    ("aex_sp_key_ranges", C.c_int, [C.c_int, C.c_int, C.c_int, C.c_int]),
    ("aex_sp_plan", C.c_int, [C.c_int, C.c_int, _VP, C.c_int]),
    ("aex_selftest_umma", C.c_int, [_VP, C.c_int, _VP, _VP, C.c_int, _VP, _VP]),
    ("aex_selftest_wait", C.c_int, [_VP, C.c_int, _VP]),
]

_lib = None
_lock = threading.Lock()


def declared_symbols() -> list[str]:
    return [s[0] for s in _SIGNATURES]


def lib() -> C.CDLL:
    """Load libaestrix_cuda.so from the package directory (raises if absent)."""
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise ImportError(
                    f"{LIB_PATH} not found: build it with `make -C aestrix_b200/csrc` "
                    "or __graft_entry__.build(); there is no CPU fallback")
            handle = C.CDLL(LIB_PATH, mode=C.RTLD_GLOBAL)
            for name, res, args in _SIGNATURES:
                fn = getattr(handle, name, None)
                if fn is None:  # reported by tests/test_capi_symbols.py
                    continue
                fn.restype = res
                fn.argtypes = args
            _lib = handle
        return _lib


def check(ctx, code: int) -> None:
    if code != AEX_OK:
        msg = lib().aex_last_error_string(ctx)
        raise AexError(code, msg.decode() if msg else "")


class Context:
    """Owns an aex_ctx for one CUDA device (mirrors the engine objects of the
    reference that own a device, e.g. DirectDiTStep)."""

    def __init__(self, device: int = 0):
        L = lib()
        h = C.c_void_p()
        rc = L.aex_ctx_create(device, C.byref(h))
        if rc != AEX_OK:
            raise AexError(rc, L.aex_last_error_string(None).decode())
        self.handle = h
        self.device = device

    def close(self):
        if getattr(self, "handle", None):
            lib().aex_ctx_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def check(self, code: int) -> None:
        check(self.handle, code)

    def sync(self, stream=None, timeout_ms: int = 30000):
        self.check(lib().aex_sync(self.handle, stream, timeout_ms))

    def device_status(self) -> int:
        v = C.c_int(0)
        self.check(lib().aex_device_status(self.handle, C.byref(v)))
        return v.value

    @property
    def sm_count(self) -> int:
        return lib().aex_device_sm_count(self.handle)


_contexts: dict[int, Context] = {}


def context(device: int = 0) -> Context:
    """Process-wide default context per device."""
    with _lock:
        ctx = _contexts.get(device)
    if ctx is None:
        ctx = Context(device)
        with _lock:
            _contexts[device] = ctx
    return ctx
