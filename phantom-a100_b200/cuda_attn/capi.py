"""ctypes view of the C ABI (include/phantom_attn.h), for callers that want the library without the
PyTorch extension: the torch-free boundary a foreign-language binding would use.

    from cuda_attn.capi import CAPI
    lib = CAPI()
    lib.fused_tc(q, k, v, o, causal=False)      # torch CUDA tensors, or raw pointers via lib.call()
"""
from __future__ import annotations

import ctypes
import os
import re

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libphantom_attn.so")

F32, F16, BF16 = 0, 1, 2
OK, ERR_INVALID, ERR_UNSUPPORTED, ERR_CUDA, ERR_DEVICE = 0, 1, 2, 3, 4

_P = ctypes.c_void_p
_I = ctypes.c_int
# name -> (restype, argtypes); mirrors include/phantom_attn.h
SIGNATURES = {
    "phantom_attn_version": (_I, []),
    "phantom_attn_last_error": (ctypes.c_char_p, []),
    "phantom_attn_fused_tc": (_I, [_P, _P, _P, _P, _I, _I, _I, _I, _I, _P]),
    "phantom_attn_fused_tc_noalloc": (_I, [_P, _P, _P, _P, _I, _I, _I, _I, _I, _P]),
    "phantom_attn_fused_tuned": (_I, [_P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _I, _P]),
    "phantom_attn_fused": (_I, [_P, _P, _P, _P, _I, _I, _I, _I, _I, _P]),
    "phantom_attn_naive": (_I, [_P, _P, _P, _P, _I, _I, _I, _I, _I, _P]),
    "phantom_attn_tiled": (_I, [_P, _P, _P, _P, _I, _I, _I, _I, _I, _P]),
    "phantom_attn_device_status": (_I, [ctypes.POINTER(ctypes.c_int)]),
    "phantom_attn_wait_expiry_probe": (_I, [_P]),
    "phantom_attn_launch_count": (ctypes.c_longlong, [_I]),
    "phantom_attn_kernel_timing": (_I, [_I]),
    "phantom_attn_kernel_timing_read": (_I, [ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_longlong)]),
    "phantom_attn_set_launch_shape": (_I, [ctypes.c_longlong, _I]),
    "phantom_attn_get_launch_shape": (_I, [ctypes.POINTER(ctypes.c_longlong), ctypes.POINTER(_I)]),
    "phantom_attn_scratch_bytes": (_I, [ctypes.POINTER(ctypes.c_longlong), ctypes.POINTER(ctypes.c_longlong), _I]),
    "phantom_attn_set_kv_parts": (_I, [_I]),
    "phantom_attn_get_kv_parts": (_I, []),
}


def header_symbols(header_path: str) -> list[str]:
    """Every function name declared in a C header (`type name(` at statement start)."""
    text = open(header_path).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"^\s*[\w\s\*]*?\b(phantom_attn_\w+)\s*\(", text, flags=re.M)))


class CapiError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(message)
        self.code = code


class CAPI:
    """Loaded libphantom_attn.so with typed entry points."""

    def __init__(self, path: str = LIB_PATH):
        if not os.path.exists(path):
            raise ImportError(f"{path} is not built; run `python phantom-a100_b200/build.py`")
        self.lib = ctypes.CDLL(path)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(self.lib, name)
            fn.restype = res
            fn.argtypes = args

    def last_error(self) -> str:
        return self.lib.phantom_attn_last_error().decode()

    def _check(self, rc: int) -> None:
        if rc != OK:
            raise CapiError(rc, self.last_error())

    # ---- torch-tensor conveniences (torch is imported lazily; the ABI itself needs no torch)
    @staticmethod
    def _dtype_code(t) -> int:
        import torch
        return {torch.float32: F32, torch.float16: F16, torch.bfloat16: BF16}[t.dtype]

    @staticmethod
    def _stream(stream):
        import torch
        if stream is None:
            stream = torch.cuda.current_stream()
        return ctypes.c_void_p(stream.cuda_stream)

    def _run(self, fn, q, k, v, o, causal, stream, *extra):
        B, H, N, d = q.shape
        rc = fn(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), B * H, N, d, self._dtype_code(q),
                int(bool(causal)), *extra, self._stream(stream))
        self._check(rc)
        return o

    def fused_tc(self, q, k, v, o, causal=False, stream=None):
        return self._run(self.lib.phantom_attn_fused_tc, q, k, v, o, causal, stream)

    def fused_tc_noalloc(self, q, k, v, o, causal=False, stream=None):
        """fused_tc without device allocation (static scratch; bf16 limited to B*H*N*d <~ 33.5M)."""
        return self._run(self.lib.phantom_attn_fused_tc_noalloc, q, k, v, o, causal, stream)

    def fused_tuned(self, q, k, v, o, causal=False, double_buffer=True, br=64, bc=32, stream=None):
        B, H, N, d = q.shape
        rc = self.lib.phantom_attn_fused_tuned(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), B * H, N, d,
                                               self._dtype_code(q), int(bool(causal)), int(bool(double_buffer)),
                                               br, bc, self._stream(stream))
        self._check(rc)
        return o

    def fused(self, q, k, v, o, causal=False, stream=None):
        return self._run(self.lib.phantom_attn_fused, q, k, v, o, causal, stream)

    def naive(self, q, k, v, o, causal=False, stream=None):
        return self._run(self.lib.phantom_attn_naive, q, k, v, o, causal, stream)

    def tiled(self, q, k, v, o, causal=False, stream=None):
        return self._run(self.lib.phantom_attn_tiled, q, k, v, o, causal, stream)

    def device_status(self) -> int:
        st = ctypes.c_int(0)
        rc = self.lib.phantom_attn_device_status(ctypes.byref(st))
        if rc not in (OK, ERR_DEVICE):
            raise CapiError(rc, self.last_error())
        return st.value

    def wait_expiry_probe(self, stream=None) -> None:
        """Launch the kernel whose bounded wait must expire (about a second); device_status() then
        reports STATUS_PROBE."""
        self._check(self.lib.phantom_attn_wait_expiry_probe(self._stream(stream)))

    def scratch_bytes(self, reset: bool = False) -> tuple[int, int]:
        """(high-water bytes of the library's per-launch scratch on the current device since the last reset,
        bytes its pool holds now)."""
        hw, rs = ctypes.c_longlong(0), ctypes.c_longlong(0)
        self._check(self.lib.phantom_attn_scratch_bytes(ctypes.byref(hw), ctypes.byref(rs), int(bool(reset))))
        return hw.value, rs.value

    def launch_count(self, reset: bool = False) -> int:
        return int(self.lib.phantom_attn_launch_count(int(reset)))

    def kernel_timing(self, enable: bool) -> None:
        self._check(self.lib.phantom_attn_kernel_timing(int(enable)))

    def kernel_timing_read(self) -> tuple[float, int]:
        """(summed milliseconds, launches) of the tensor-core kernel since timing was enabled."""
        ms, n = ctypes.c_double(0.0), ctypes.c_longlong(0)
        self._check(self.lib.phantom_attn_kernel_timing_read(ctypes.byref(ms), ctypes.byref(n)))
        return ms.value, n.value

    def set_launch_shape(self, l2_group_kib: int = 0, max_ctas: int = 0) -> None:
        """Launch-shape override of the tensor-core kernel on the calling thread (0 = automatic)."""
        self._check(self.lib.phantom_attn_set_launch_shape(int(l2_group_kib), int(max_ctas)))

    def set_kv_parts(self, allow: bool) -> None:
        """Whether a last partial wave may be cut into K/V parts (calling thread; default True). False keeps
        results bit-identical for every launch shape and GPU count."""
        self._check(self.lib.phantom_attn_set_kv_parts(int(bool(allow))))

    def get_kv_parts(self) -> bool:
        return bool(self.lib.phantom_attn_get_kv_parts())

    def get_launch_shape(self) -> tuple[int, int]:
        """(l2_group_kib, max_ctas) of the calling thread; 0 = automatic."""
        kib, ctas = ctypes.c_longlong(0), ctypes.c_int(0)
        self._check(self.lib.phantom_attn_get_launch_shape(ctypes.byref(kib), ctypes.byref(ctas)))
        return kib.value, ctas.value
