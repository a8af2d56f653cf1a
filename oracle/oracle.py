"""ctypes front of the CPU oracle (liborc.so, built from oracle/sage_ref.cpp by oracle/Makefile).

TEST INFRASTRUCTURE ONLY: the checker that tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg use.
Nothing in the product imports this module.

Every function takes and returns numpy arrays; an input may also be ``(array, element_offset)`` to point inside a wider
buffer (q, k, v inside one qkv buffer of row stride 3*H*D). Element-type codes follow ``kernels/h3sycl.h:21`` of the reference
(0 = float32, 1 = float16, 2 = bfloat16); float16/bfloat16 arrays are passed as their uint16 bit patterns.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liborc.so")
F32, F16, BF16 = 0, 1, 2
BLOCK = 64  # quantisation block (kernels/h3sycl.cpp:1681)

_lib = None


def build() -> str:
    """Compiles liborc.so with oracle/Makefile (a no-op when it is current), and oracle/_ref/libref.so from the
    reference's own source where that source is present (oracle/ref_build.py)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    import importlib.util

    spec = importlib.util.spec_from_file_location("ref_build", os.path.join(HERE, "ref_build.py"))
    rb = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(rb)
    if rb.available():
        rb.build()
    return LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        P, I64, I = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
        for name in ("orc_f32_to_f16", "orc_f16_to_f32", "orc_f32_to_bf16", "orc_bf16_to_f32"):
            getattr(L, name).argtypes = [P, P, I64]
            getattr(L, name).restype = None
        L.orc_threads.restype = I
        L.orc_set_threads.argtypes = [I]
        L.orc_kmean.argtypes = [P, I, I64, I64, I64, I64, P]
        L.orc_quant.argtypes = [P, I, I64, I64, I64, I64, P, P, P]
        L.orc_sage_prepass.argtypes = [P, P, P, I, I64, I64, I64, I64, P, P, P, P]
        L.orc_sage_rows.argtypes = [P, P, P, P, P, I64, I64, I64, ctypes.c_float, P, P, I64, P]
        L.orc_sdpa_rows.argtypes = [P, P, P, I, I64, I64, I64, I64, P, P, I64, P]
        L.orc_exact_rows.argtypes = [P, P, P, I, I64, I64, I64, I64, P, P, I64, P]
        L.orc_attention.argtypes = [P, P, P, I, I64, I64, I64, I64, P, I, I64]
        L.orc_attention.restype = I
        L.orc_rms_rope.argtypes = [P, I, I64, I64, I64, I64, P, ctypes.c_float, P, I]
        L.orc_rms_rope.restype = I
        L.orc_attention_causal.argtypes = [P, P, P, I, I64, I64, I64, I64, I64, I64, P]
        L.orc_attention_causal.restype = I
        L.orc_rotq.argtypes = [P, I, I64, I64, I, P, P]
        L.orc_int8_linear.argtypes = [P, I, I64, I64, P, I64, P, I64, P, P, I, I]
        L.orc_int8_linear_dense.argtypes = [P, I64, I64, P, I64, P, I64, P, I, P]
        _lib = L
    return _lib


def _p(a):
    """Address of an array, or of element `off` of it when given as (array, off)."""
    if a is None:
        return None
    off = 0
    if isinstance(a, tuple):
        a, off = a
    assert a.flags["C_CONTIGUOUS"], "oracle arrays must be C-contiguous"
    return a.ctypes.data + int(off) * a.itemsize


def threads() -> int:
    return lib().orc_threads()


def set_threads(n: int) -> None:
    lib().orc_set_threads(int(n))


# ---- dtype helpers ---------------------------------------------------------------------------------------------------
def f32_to_f16(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty(x.shape, np.uint16)
    lib().orc_f32_to_f16(_p(x), _p(y), x.size)
    return y


def f16_to_f32(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.uint16)
    y = np.empty(x.shape, np.float32)
    lib().orc_f16_to_f32(_p(x), _p(y), x.size)
    return y


def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty(x.shape, np.uint16)
    lib().orc_f32_to_bf16(_p(x), _p(y), x.size)
    return y


def bf16_to_f32(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.uint16)
    y = np.empty(x.shape, np.float32)
    lib().orc_bf16_to_f32(_p(x), _p(y), x.size)
    return y


def _dt_of(x: np.ndarray) -> int:
    if x.dtype == np.float32:
        return F32
    raise TypeError("pass float16/bfloat16 data as uint16 bits together with an explicit dt")


# ---- the Sage pre-pass -------------------------------------------------------------------------------------------------
def kmean(k: np.ndarray, dt: int, S: int, H: int, D: int, stride: int) -> np.ndarray:
    out = np.empty(H * D, np.float32)
    lib().orc_kmean(_p(k), dt, S, H, D, stride, _p(out))
    return out


def quant(x: np.ndarray, dt: int, S: int, H: int, D: int, stride: int, mean: np.ndarray | None = None):
    nb = (S + BLOCK - 1) // BLOCK
    dst = np.empty((H, S, D), np.int8)
    sc = np.empty((H, nb), np.float32)
    lib().orc_quant(_p(x), dt, S, H, D, stride, _p(mean), _p(dst), _p(sc))
    return dst, sc


def sage_prepass(q, k, v, dt: int, S: int, H: int, D: int, stride: int):
    """Returns (iq int8 [H,S,D], ik int8 [H,S,D], qs [H,nb], ks [H,nb], kmean [H*D], hv uint16 [H,S,D])."""
    nb = (S + BLOCK - 1) // BLOCK
    iq = np.empty((H, S, D), np.int8)
    ik = np.empty((H, S, D), np.int8)
    sc = np.empty(2 * H * nb + H * D, np.float32)
    hv = np.empty((H, S, D), np.uint16)
    lib().orc_sage_prepass(_p(q), _p(k), _p(v), dt, S, H, D, stride, _p(iq), _p(ik), _p(sc), _p(hv))
    return iq, ik, sc[: H * nb].reshape(H, nb).copy(), sc[H * nb: 2 * H * nb].reshape(H, nb).copy(), \
        sc[2 * H * nb:].copy(), hv


def _rows(rows_h, rows_s):
    rh = np.ascontiguousarray(rows_h, dtype=np.int64)
    rs = np.ascontiguousarray(rows_s, dtype=np.int64)
    assert rh.shape == rs.shape
    return rh, rs


def sage_rows(iq, ik, hv, qs, ks, S, H, D, rows_h, rows_s, scale: float | None = None) -> np.ndarray:
    """Sage-semantics output rows (half bits [n, D]) for (head, token) pairs."""
    rh, rs = _rows(rows_h, rows_s)
    out = np.empty((rh.size, D), np.uint16)
    sc = float(np.float32(1.0) / np.sqrt(np.float32(D))) if scale is None else scale
    lib().orc_sage_rows(_p(iq), _p(ik), _p(hv), _p(np.ascontiguousarray(qs, np.float32)),
                        _p(np.ascontiguousarray(ks, np.float32)), S, H, D, sc, _p(rh), _p(rs), rh.size, _p(out))
    return out


def sdpa_rows(q, k, v, dt, S, H, D, stride, rows_h, rows_s) -> np.ndarray:
    """fp16 fused-SDPA-semantics output rows (half bits [n, D])."""
    rh, rs = _rows(rows_h, rows_s)
    out = np.empty((rh.size, D), np.uint16)
    lib().orc_sdpa_rows(_p(q), _p(k), _p(v), dt, S, H, D, stride, _p(rh), _p(rs), rh.size, _p(out))
    return out


def exact_rows(q, k, v, dt, S, H, D, stride, rows_h, rows_s) -> np.ndarray:
    """float64 softmax attention rows (float32 [n, D]): the tolerance anchor."""
    rh, rs = _rows(rows_h, rows_s)
    out = np.empty((rh.size, D), np.float32)
    lib().orc_exact_rows(_p(q), _p(k), _p(v), dt, S, H, D, stride, _p(rh), _p(rs), rh.size, _p(out))
    return out


def attention(q, k, v, dt, S, H, D, stride, out_dt=F16, sage_min_s=8192) -> np.ndarray:
    """h3s_attention semantics: out [S, H*D] in out_dt (uint16 bits for half/bf16, float32 for F32)."""
    out = np.empty((S, H * D), np.float32 if out_dt == F32 else np.uint16)
    rc = lib().orc_attention(_p(q), _p(k), _p(v), dt, S, H, D, stride, _p(out), out_dt, sage_min_s)
    if rc != 0:
        raise ValueError("orc_attention: the row stride is shorter than a row")
    return out


# ---- comparison, as the reference defines it (engine/h3-core/src/reference.rs:85-95) --------------------------------
def compare(a: np.ndarray, b: np.ndarray) -> tuple[float, float]:
    """(relative error |a-b|/|b|, cosine) over the whole arrays, in float64."""
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    d2 = float(np.sum((a - b) ** 2))
    a2 = float(np.sum(a * a))
    b2 = float(np.sum(b * b))
    ab = float(np.sum(a * b))
    return (d2 / max(b2, 1e-300)) ** 0.5, ab / max((a2 ** 0.5) * (b2 ** 0.5), 1e-300)


def row_cosines(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """Cosine per row of two [n, D] arrays, in float64."""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    num = np.sum(a * b, axis=1)
    den = np.maximum(np.linalg.norm(a, axis=1) * np.linalg.norm(b, axis=1), 1e-300)
    return num / den


def rms_rope(x: np.ndarray, dt: int, M: int, H: int, D: int, stride: int, weight: np.ndarray, eps: float,
             cs: np.ndarray, rot_dim: int) -> np.ndarray:
    """Per-head RMS norm + rotary rotation (kernels/h3sycl.cpp:1276-1376) on a copy of x; returns the copy. x holds the
    element bits (uint16 for half/bfloat16, float32 for float) of M rows at element stride `stride`."""
    y = np.array(x, copy=True)
    w = np.ascontiguousarray(weight, np.float32)
    c = np.ascontiguousarray(cs, np.float32)
    rc = lib().orc_rms_rope(_p(y), dt, M, H, D, stride, _p(w), ctypes.c_float(eps), _p(c), rot_dim)
    if rc != 0:
        raise ValueError("rms_rope: rot_dim must be even, at most D, leave an even remainder; stride >= H*D")
    return y


def attention_causal(q, k, v, dt: int, L: int, Hq: int, Hkv: int, D: int, qs: int, kvs: int) -> np.ndarray:
    """Causal attention with grouped heads (kernels/h3sycl.cpp:870-898): q rows of stride qs, k and v rows of stride kvs
    (element bits of type dt; each argument may be an (array, element offset) pair); returns out [L, Hq*D] in dt bits."""
    base = q[0] if isinstance(q, tuple) else q
    out = np.zeros((L, Hq * D), dtype=base.dtype)
    rc = lib().orc_attention_causal(_p(q), _p(k), _p(v), dt, L, Hq, Hkv, D, qs, kvs, _p(out))
    if rc != 0:
        raise ValueError("attention_causal: D <= 256 and Hq a multiple of Hkv")
    return out


def rotq(x, dt: int, M: int, K: int, group: int):
    """ConvRot rotation + per-row int8 quantisation (kernels/h3sycl.cpp:404-470 order): returns (xq [M, K] int8, rs [M])."""
    xq = np.zeros((M, K), np.int8)
    rs = np.zeros(M, np.float32)
    lib().orc_rotq(_p(x), dt, M, K, group, _p(xq), _p(rs))
    return xq, rs


def int8_linear(x, dt: int, M: int, K: int, w: np.ndarray, N: int, wscale, bias, out_dt: int, group: int) -> np.ndarray:
    """The int8 ConvRot linear (kernels/h3sycl.h:74-85, the fused kernel's rotation order): x [M, K] as element bits
    of type dt; out [M, N] as bits (uint16) for F16/BF16, float32 for F32."""
    out = np.zeros((M, N), np.float32 if out_dt == F32 else np.uint16)
    ws = np.ascontiguousarray(wscale, np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, np.float32)
    lib().orc_int8_linear(_p(np.ascontiguousarray(x)), dt, M, K, _p(np.ascontiguousarray(w, np.int8)), N, _p(ws), ws.size,
                          _p(b), _p(out), out_dt, group)
    return out


def int8_linear_dense(x: np.ndarray, M: int, K: int, w: np.ndarray, N: int, wscale, bias, group: int) -> np.ndarray:
    """engine/h3-core/src/reference.rs:37-82 as written (dense Hadamard product); x float32 [M, K]; out float32 [M, N]."""
    out = np.zeros((M, N), np.float32)
    ws = np.ascontiguousarray(wscale, np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, np.float32)
    lib().orc_int8_linear_dense(_p(np.ascontiguousarray(x, np.float32)), M, K, _p(np.ascontiguousarray(w, np.int8)), N,
                                _p(ws), ws.size, _p(b), group, _p(out))
    return out


# ---- the reference's own source, compiled for the CPU (oracle/_ref/libref.so, built by oracle/ref_build.py) ---------
# These run kernels/h3sycl.cpp:38-63, 1276-1376, 1733-1771 of the reference unchanged (through oracle/ref_shim.h), so
# the restatement above and the GPU kernels can be compared with the reference itself. The library is built where the
# reference's source is present and travels with the other built files; ref_available() is False without it.
REF_LIB_PATH = os.path.join(HERE, "_ref", "libref.so")
_ref = None


def ref_available() -> bool:
    return os.path.exists(REF_LIB_PATH)


def ref_lib() -> ctypes.CDLL:
    global _ref
    if _ref is None:
        if not ref_available():
            raise FileNotFoundError(f"{REF_LIB_PATH} is missing: build it with oracle/ref_build.py where the "
                                    "reference's source is present")
        L = ctypes.CDLL(REF_LIB_PATH)
        P, I64, I = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
        L.ref_load.argtypes = [P, I, ctypes.c_uint64]
        L.ref_load.restype = ctypes.c_float
        L.ref_store.argtypes = [P, I, ctypes.c_uint64, ctypes.c_float]
        L.ref_store.restype = None
        L.ref_sage_prepass.argtypes = [P, P, P, I, I64, I64, I64, I64, P, P, P, P]
        L.ref_sage_prepass.restype = None
        L.ref_out_relayout.argtypes = [P, P, I, I64, I64, I64]
        L.ref_out_relayout.restype = None
        L.ref_rms_rope.argtypes = [P, I, I64, I64, I64, I64, P, ctypes.c_float, P, I]
        L.ref_rms_rope.restype = I
        L.ref_error.restype = ctypes.c_char_p
        _ref = L
    return _ref


def ref_sage_prepass(q, k, v, dt: int, S: int, H: int, D: int, stride: int):
    """The reference's pre-pass (kernels/h3sycl.cpp:1733-1764) as compiled from its source: same returns as
    sage_prepass (iq, ik, qs, ks, kmean, hv)."""
    nb = (S + BLOCK - 1) // BLOCK
    iq = np.empty((H, S, D), np.int8)
    ik = np.empty((H, S, D), np.int8)
    sc = np.empty(2 * H * nb + H * D, np.float32)
    hv = np.empty((H, S, D), np.uint16)
    ref_lib().ref_sage_prepass(_p(q), _p(k), _p(v), dt, S, H, D, stride, _p(iq), _p(ik), _p(sc), _p(hv))
    return iq, ik, sc[: H * nb].reshape(H, nb).copy(), sc[H * nb: 2 * H * nb].reshape(H, nb).copy(), \
        sc[2 * H * nb:].copy(), hv


def ref_out_relayout(ao_bits: np.ndarray, out_dt: int, S: int, H: int, D: int) -> np.ndarray:
    """kernels/h3sycl.cpp:1769-1771 from the reference's source: half [H, S, D] -> out_dt [S, H*D] (bits)."""
    out = np.empty((S, H * D), np.float32 if out_dt == F32 else np.uint16)
    ref_lib().ref_out_relayout(_p(np.ascontiguousarray(ao_bits, np.uint16)), _p(out), out_dt, S, H, D)
    return out


def ref_load(x: np.ndarray, dt: int) -> np.ndarray:
    """kernels/h3sycl.cpp:49-55 (load) from the reference's source, element by element."""
    x = np.ascontiguousarray(x)
    L = ref_lib()
    return np.array([L.ref_load(_p(x), dt, i) for i in range(x.size)], np.float32)


def ref_store(v: np.ndarray, dt: int) -> np.ndarray:
    """kernels/h3sycl.cpp:56-62 (store) from the reference's source: float32 values -> element bits of type dt."""
    v = np.ascontiguousarray(v, np.float32)
    out = np.empty(v.shape, np.float32 if dt == F32 else np.uint16)
    L = ref_lib()
    for i in range(v.size):
        L.ref_store(_p(out), dt, i, float(v.flat[i]))
    return out


def ref_rms_rope(x: np.ndarray, dt: int, M: int, H: int, D: int, stride: int, weight: np.ndarray, eps: float,
                 cs: np.ndarray, rot_dim: int) -> np.ndarray:
    """h3s_rms_rope (kernels/h3sycl.cpp:1276-1376) from the reference's source on a copy of x (its rsqrt correctly
    rounded: SYCL leaves rsqrt's accuracy to the implementation)."""
    y = np.array(x, copy=True)
    rc = ref_lib().ref_rms_rope(_p(y), dt, M, H, D, stride, _p(np.ascontiguousarray(weight, np.float32)),
                                ctypes.c_float(eps), _p(np.ascontiguousarray(cs, np.float32)), rot_dim)
    if rc != 0:
        raise ValueError(ref_lib().ref_error().decode())
    return y
