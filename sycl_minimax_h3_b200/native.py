"""ctypes bindings of libh3cuda.so (include/h3cuda.h) and libh3sage.so (include/h3sage.h).

These are the thin FFI bindings the reference's ``engine/h3-sys/src/lib.rs`` holds for libh3sycl.so, for Python: every
symbol is resolved when the library is loaded, and a missing library or symbol is an error (there is no fallback of
any kind). Errors follow the ABI: an int return of -1 raises ``H3Error`` with ``h3s_last_error()``.
"""
from __future__ import annotations

import ctypes
import os

LIB_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "lib")
CUDA_LIB = os.path.join(LIB_DIR, "libh3cuda.so")
SAGE_LIB = os.path.join(LIB_DIR, "libh3sage.so")

F32, F16, BF16 = 0, 1, 2  # kernels/h3sycl.h:21

P, I, I64, U64 = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_uint64

# (name, restype, argtypes): every entry point of include/h3cuda.h
CUDA_SYMBOLS = [
    ("h3s_last_error", ctypes.c_char_p, []),
    ("h3s_open", P, []),
    ("h3s_gpu_count", I, []),
    ("h3s_gpu_info", I, [I, ctypes.c_char_p, I, ctypes.POINTER(U64), ctypes.c_char_p, I]),
    ("h3s_open_gpu", P, [I]),
    ("h3s_create", P, [P]),
    ("h3s_destroy", None, [P]),
    ("h3s_device_name", ctypes.c_char_p, [P]),
    ("h3s_alloc", P, [P, U64]),
    ("h3s_free", None, [P, P]),
    ("h3s_mem_used", U64, [P]),
    ("h3s_mem_cap", U64, [P]),
    ("h3s_mem_free", U64, [P]),
    ("h3s_write", I, [P, P, P, U64]),
    ("h3s_read", I, [P, P, P, U64]),
    ("h3s_copy", I, [P, P, P, U64]),
    ("h3s_wait", I, [P]),
    ("h3s_alloc_host", P, [P, U64]),
    ("h3s_free_host", None, [P, P]),
    ("h3s_upload", I, [P, P, P, U64]),
    ("h3s_upload_wait", I, [P]),
    ("h3s_attention", I, [P, P, P, P, I, I64, I64, I64, I64, P, I]),
    ("h3s_attention_batch", I, [P, P, P, P, I, I64, I64, I64, I64, I64, P, I]),
    ("h3s_rms_rope", I, [P, P, I, I64, I64, I64, I64, P, ctypes.c_float, P, I]),
    ("h3s_attention_causal", I, [P, P, P, P, I, I64, I64, I64, I64, I64, I64, P]),
    ("h3s_int8_linear", I, [P, P, I, I64, I64, P, I64, P, I64, P, P, I, I]),
    ("h3s_ipc_handle", I, [P, P, P]),
    ("h3s_ipc_open", P, [P, P]),
    ("h3s_ipc_close", I, [P, P]),
    ("h3s_ulysses_push_qkv", I, [P, P, I64, I64, I64, I, I, I, P]),
    ("h3s_ulysses_push_out", I, [P, P, I64, I64, I64, I, I, I, P]),
    ("h3s_attention_ulysses", I, [P, P, P, P, I, I64, I64, I64, I64, P, I, I, I]),
    ("h3s_sage_prepass", I, [P, P, P, I, I64, I64, I64, I64, P, P, P]),
    ("h3s_sage_prepass_rope", I, [P, P, P, I, I64, I64, I64, I64, P, P, ctypes.c_float, P, I, P, P, P]),
    ("h3s_attention_rms_rope", I, [P, P, P, P, I, I64, I64, I64, I64, P, I, P, P, ctypes.c_float, P, I]),
    ("h3s_stream", P, [P]),
    ("h3s_selftest_wait_timeout", I, [P, U64]),
    ("h3s_attention_sage_static", I, [P, P, P, P, I64, I64, I64, I64, P, I, P]),
]
# every entry point of include/h3sage.h
SAGE_SYMBOLS = [
    ("h3sage_error", ctypes.c_char_p, []),
    ("h3sage_attention", I, [P, P, P, P, P, P, P, I, I64, I64, I64, ctypes.c_float]),
    ("h3sage_attention_strided", I, [P, P, P, P, I64, I64, P, I, I64, I64, P, P, I, I64, I64, I64, ctypes.c_float, P, U64]),
    ("h3sage_attention_peers", I, [P, P, P, P, I64, I64, P, I, I, I64, I64, P, P, I, I64, I64, I64, ctypes.c_float, P,
                                   U64]),
    ("h3sage_check", I, [P]),
]


class H3Error(RuntimeError):
    pass


_libs: dict[str, ctypes.CDLL] = {}


def _load(path: str, symbols) -> ctypes.CDLL:
    if path in _libs:
        return _libs[path]
    if not os.path.exists(path):
        raise H3Error(f"{path} is missing: build it first (python -c 'import __graft_entry__ as g; g.build()')")
    L = ctypes.CDLL(path, mode=ctypes.RTLD_LOCAL)
    for name, res, args in symbols:
        fn = getattr(L, name)  # AttributeError when the symbol is missing: the library is not this ABI
        fn.restype = res
        fn.argtypes = args
    _libs[path] = L
    return L


def lib() -> ctypes.CDLL:
    """libh3cuda.so with every include/h3cuda.h entry point resolved."""
    return _load(CUDA_LIB, CUDA_SYMBOLS)


def sage_lib() -> ctypes.CDLL:
    """libh3sage.so with every include/h3sage.h entry point resolved."""
    return _load(SAGE_LIB, SAGE_SYMBOLS)


def last_error() -> str:
    return (lib().h3s_last_error() or b"").decode(errors="replace")


def check(rc: int, what: str = "") -> None:
    if rc != 0:
        raise H3Error(f"{what}: {last_error()}" if what else last_error())


def dt_code(dtype) -> int:
    """kernels/h3sycl.h element-type code of a torch dtype."""
    import torch

    if dtype == torch.float16:
        return F16
    if dtype == torch.bfloat16:
        return BF16
    if dtype == torch.float32:
        return F32
    raise H3Error(f"{dtype} is not a floating-point tensor type of the ABI (float32, float16, bfloat16)")


class Context:
    """An h3s context. ``Context()`` wraps PyTorch's current CUDA stream (h3s_create), so calls are ordered with PyTorch's
    own work and torch tensors' device pointers are valid; ``Context.open_gpu(i)`` owns a stream on GPU i (h3s_open_gpu)."""

    def __init__(self, stream=None, *, _handle=None):
        self._lib = lib()
        if _handle is not None:
            self.handle = _handle
        else:
            import torch

            s = torch.cuda.current_stream() if stream is None else stream
            raw = ctypes.c_void_p(int(s.cuda_stream) if hasattr(s, "cuda_stream") else int(s))
            self._stream_box = raw  # the pointer h3s_create reads from
            self.handle = self._lib.h3s_create(ctypes.byref(raw))
        if not self.handle:
            raise H3Error(f"h3s context: {last_error()}")

    @classmethod
    def open_gpu(cls, index: int = 0) -> "Context":
        h = lib().h3s_open_gpu(index)
        if not h:
            raise H3Error(f"h3s_open_gpu({index}): {last_error()}")
        return cls(_handle=h)

    def close(self) -> None:
        if self.handle:
            self._lib.h3s_destroy(self.handle)
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ---- device memory and copies ----
    @property
    def device_name(self) -> str:
        return self._lib.h3s_device_name(self.handle).decode()

    def alloc(self, nbytes: int) -> int:
        p = self._lib.h3s_alloc(self.handle, nbytes)
        if not p:
            raise H3Error(f"h3s_alloc: {last_error()}")
        return p

    def free(self, p: int) -> None:
        self._lib.h3s_free(self.handle, p)

    def mem_used(self) -> int:
        return self._lib.h3s_mem_used(self.handle)

    def mem_cap(self) -> int:
        return self._lib.h3s_mem_cap(self.handle)

    def write(self, dst: int, src_host: int, nbytes: int) -> None:
        check(self._lib.h3s_write(self.handle, dst, src_host, nbytes), "h3s_write")

    def read(self, dst_host: int, src: int, nbytes: int) -> None:
        check(self._lib.h3s_read(self.handle, dst_host, src, nbytes), "h3s_read")

    def wait(self) -> None:
        check(self._lib.h3s_wait(self.handle), "h3s_wait")

    @property
    def stream(self) -> int:
        return self._lib.h3s_stream(self.handle) or 0

    # ---- attention (raw pointers) ----
    def attention(self, q: int, k: int, v: int, dt: int, S: int, H: int, D: int, stride: int, out: int, out_dt: int) -> None:
        check(self._lib.h3s_attention(self.handle, q, k, v, dt, S, H, D, stride, out, out_dt), "h3s_attention")

    def attention_batch(self, q: int, k: int, v: int, dt: int, B: int, S: int, H: int, D: int, stride: int, out: int,
                        out_dt: int) -> None:
        check(self._lib.h3s_attention_batch(self.handle, q, k, v, dt, B, S, H, D, stride, out, out_dt),
              "h3s_attention_batch")

    def rms_rope(self, x: int, dt: int, M: int, H: int, D: int, stride: int, weight: int, eps: float, cs: int,
                 rot_dim: int) -> None:
        check(self._lib.h3s_rms_rope(self.handle, x, dt, M, H, D, stride, weight, eps, cs, rot_dim), "h3s_rms_rope")

    def int8_linear(self, x: int, x_dt: int, M: int, K: int, w: int, N: int, wscale: int, n_wscale: int, bias: int,
                    out: int, out_dt: int, group: int) -> None:
        check(self._lib.h3s_int8_linear(self.handle, x, x_dt, M, K, w, N, wscale, n_wscale, bias, out, out_dt, group),
              "h3s_int8_linear")

    def ipc_handle(self, ptr: int) -> bytes:
        buf = ctypes.create_string_buffer(64)
        check(self._lib.h3s_ipc_handle(self.handle, ptr, ctypes.cast(buf, ctypes.c_void_p)), "h3s_ipc_handle")
        return buf.raw

    def ipc_open(self, handle: bytes) -> int:
        if len(handle) != 64:
            raise H3Error("h3s_ipc_open: a handle is 64 bytes")
        buf = ctypes.create_string_buffer(handle, 64)
        p = self._lib.h3s_ipc_open(self.handle, ctypes.cast(buf, ctypes.c_void_p))
        if not p:
            raise H3Error(f"h3s_ipc_open: {last_error()}")
        return p

    def ipc_close(self, ptr: int) -> None:
        check(self._lib.h3s_ipc_close(self.handle, ptr), "h3s_ipc_close")

    def ulysses_push_qkv(self, shard: int, s: int, H: int, D: int, es: int, P: int, rank: int, dst: list[int]) -> None:
        table = (ctypes.c_void_p * len(dst))(*dst)
        check(self._lib.h3s_ulysses_push_qkv(self.handle, shard, s, H, D, es, P, rank, table), "h3s_ulysses_push_qkv")

    def ulysses_push_out(self, out_heads: int, s: int, H: int, D: int, es: int, P: int, rank: int, dst: list[int]) -> None:
        table = (ctypes.c_void_p * len(dst))(*dst)
        check(self._lib.h3s_ulysses_push_out(self.handle, out_heads, s, H, D, es, P, rank, table), "h3s_ulysses_push_out")

    def attention_ulysses(self, q: int, k: int, v: int, dt: int, S: int, H: int, D: int, stride: int,
                          out_shards: list[int], P: int, rank: int, out_dt: int) -> None:
        table = (ctypes.c_void_p * len(out_shards))(*out_shards)
        check(self._lib.h3s_attention_ulysses(self.handle, q, k, v, dt, S, H, D, stride, table, P, rank, out_dt),
              "h3s_attention_ulysses")

    def attention_causal(self, q: int, k: int, v: int, dt: int, L: int, Hq: int, Hkv: int, D: int, qs: int, kvs: int,
                         out: int) -> None:
        check(self._lib.h3s_attention_causal(self.handle, q, k, v, dt, L, Hq, Hkv, D, qs, kvs, out), "h3s_attention_causal")

    def sage_prepass(self, q: int, k: int, dt: int, S: int, H: int, D: int, stride: int, iq: int, ik: int, sc: int) -> None:
        check(self._lib.h3s_sage_prepass(self.handle, q, k, dt, S, H, D, stride, iq, ik, sc), "h3s_sage_prepass")

    def sage_prepass_rope(self, q: int, k: int, dt: int, S: int, H: int, D: int, stride: int, wq: int, wk: int,
                          eps: float, cs: int, rot_dim: int, iq: int, ik: int, sc: int) -> None:
        check(self._lib.h3s_sage_prepass_rope(self.handle, q, k, dt, S, H, D, stride, wq, wk, eps, cs, rot_dim, iq, ik,
                                              sc), "h3s_sage_prepass_rope")

    def attention_rms_rope(self, q: int, k: int, v: int, dt: int, S: int, H: int, D: int, stride: int, out: int,
                           out_dt: int, wq: int, wk: int, eps: float, cs: int, rot_dim: int) -> None:
        check(self._lib.h3s_attention_rms_rope(self.handle, q, k, v, dt, S, H, D, stride, out, out_dt, wq, wk, eps, cs,
                                               rot_dim), "h3s_attention_rms_rope")

    def selftest_wait_timeout(self, wait_ns: int) -> None:
        check(self._lib.h3s_selftest_wait_timeout(self.handle, wait_ns), "h3s_selftest_wait_timeout")


def gpu_count() -> int:
    n = lib().h3s_gpu_count()
    if n < 0:
        raise H3Error(f"h3s_gpu_count: {last_error()}")
    return n


def gpu_info(index: int) -> dict:
    name = ctypes.create_string_buffer(256)
    pci = ctypes.create_string_buffer(64)
    mem = U64(0)
    check(lib().h3s_gpu_info(index, name, 256, ctypes.byref(mem), pci, 64), "h3s_gpu_info")
    return {"name": name.value.decode(), "mem_bytes": mem.value, "pci": pci.value.decode()}
