"""CPU oracle for the stereo cost-volume front end -- TEST INFRASTRUCTURE ONLY.

Python (numpy + ctypes) bindings to ``oracle/_build/libww_oracle.so``, the
plain-C restatement of the reference's CorrVolume / CostStem3D semantics in
``oracle/ww_oracle.c``, and to ``oracle/_ref/libww_ref.so``, the reference's
own CUDA kernels rebuilt for sm_100a by ``oracle/Makefile``.

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline /
reference arm of ``bench.py`` may import this package: it is the checker,
never the thing measured or shipped.  The product package
(``whirlwind_trt_plugins_b200``) does not import it and has no CPU fallback.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(_HERE, "_build", "libww_oracle.so")
REF_SO = os.path.join(_HERE, "_ref", "libww_ref.so")

SCALE_DIV = 0
SCALE_MULINV = 1
ACC_F32_SEQ = 0
ACC_F64 = 1
ACT_RELU = 0
ACT_RELU6 = 1

_lib = None
_ref = None


def build(force: bool = False) -> str:
    """Compile the C oracle with the Makefile next to this file."""
    if force or not os.path.exists(ORACLE_SO):
        subprocess.run(["make", "-C", _HERE, "all"], check=True, capture_output=True)
    return ORACLE_SO


def build_ref(src: str | None = None) -> str | None:
    """Compile the reference kernels from the reference project's src/
    directory: `src`, else $WW_REF_SRC.  Without either (or where that tree
    does not exist, as on the GPU box) the already built library is used if
    present."""
    src = src or os.environ.get("WW_REF_SRC")
    if not src or not os.path.isdir(src):
        return REF_SO if os.path.exists(REF_SO) else None
    subprocess.run(["make", "-C", _HERE, "ref", f"REF_SRC={src}"], check=True, capture_output=True)
    return REF_SO


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(ORACLE_SO)
        p, i, f = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
        L.orc_corr_f32.argtypes = [p, p, p] + [i] * 7
        L.orc_corr_f16.argtypes = [p, p, p] + [i] * 8
        L.orc_stem_ref3.argtypes = [p] * 8 + [i] * 5
        L.orc_stem.argtypes = [p, p, p, p] + [i] * 13
        L.orc_corr_stem.argtypes = [p, p, p, p, p] + [i] * 15
        L.orc_ref_corr_scale_mode.argtypes = [i] * 7
        L.orc_fold_bn.argtypes = [p, p, p, i, i, p, p]
        L.orc_fold_bn.restype = None
        L.orc_f32_to_f16.argtypes = [f]
        L.orc_f32_to_f16.restype = ctypes.c_uint16
        L.orc_f16_to_f32.argtypes = [ctypes.c_uint16]
        L.orc_f16_to_f32.restype = f
        L.orc_f32_to_f16_array.argtypes = [p, p, ctypes.c_int64]
        L.orc_f32_to_f16_array.restype = None
        L.orc_hw_threads.restype = i
        L.orc_nv12_decode.argtypes = [p] + [i] * 6 + [p, i]
        L.orc_disparity_regression.argtypes = [p] + [i] * 7 + [p, i]
        _lib = L
    return _lib


def ref_lib() -> ctypes.CDLL:
    """The reference's CUDA kernels (GPU box or a machine with a GPU)."""
    global _ref
    if _ref is None:
        if not os.path.exists(REF_SO):
            build_ref()
        if not os.path.exists(REF_SO):
            raise RuntimeError("oracle/_ref/libww_ref.so is missing; run `make -C oracle ref` "
                               "where the reference sources are available")
        R = ctypes.CDLL(REF_SO)
        p, i = ctypes.c_void_p, ctypes.c_int
        R.wwref_corr_volume_f16.argtypes = [p, p, p] + [i] * 5 + [p]
        R.wwref_corr_volume_f32.argtypes = [p, p, p] + [i] * 5 + [p]
        R.wwref_corr_volume_grouped_f16.argtypes = [p, p, p] + [i] * 6 + [p]
        R.wwref_cost_stem3d.argtypes = [p] * 8 + [i] * 4 + [p]
        R.wwref_nv12_decode_f16.argtypes = [p, p] + [i] * 4 + [p]
        R.wwref_nv12_decode_f32.argtypes = [p, p] + [i] * 4 + [p]
        _ref = R
    return _ref


def _ptr(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


def _h(a: np.ndarray) -> np.ndarray:
    """fp16 array -> its uint16 bit pattern view (C-contiguous)."""
    a = np.ascontiguousarray(a)
    if a.dtype == np.float16:
        return a.view(np.uint16)
    assert a.dtype == np.uint16, a.dtype
    return a


def _check(rc: int, what: str) -> None:
    if rc != 0:
        raise ValueError(f"oracle {what} rejected its arguments (rc={rc})")


def nthreads_default() -> int:
    return int(lib().orc_hw_threads())


def f32_to_f16(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, dtype=np.uint16)
    lib().orc_f32_to_f16_array(_ptr(x), _ptr(out), x.size)
    return out.view(np.float16)


def ref_scale_mode(is_half: bool, B: int, C: int, H: int, W: int, D: int, sm_count: int = 148) -> int:
    """Which reference CorrVolume kernel one launchCorrVolume call would use."""
    return int(lib().orc_ref_corr_scale_mode(int(is_half), B, C, H, W, D, sm_count))


def grouped_scale_mode(is_half: bool, B: int, C: int, G: int, H: int, W: int, D: int,
                       sm_count: int = 148) -> int:
    """Scale mode of the reference's group-wise composition: G == 1 is one
    call over all channels; G > 1 is one call per (batch, group) with B=1, C=C/G."""
    if G == 1:
        return ref_scale_mode(is_half, B, C, H, W, D, sm_count)
    return ref_scale_mode(is_half, 1, C // G, H, W, D, sm_count)


def corr_f32(L: np.ndarray, R: np.ndarray, D: int, G: int = 1, nthreads: int = 0) -> np.ndarray:
    L = np.ascontiguousarray(L, dtype=np.float32)
    R = np.ascontiguousarray(R, dtype=np.float32)
    B, C, H, W = L.shape
    out = np.empty((B, G, D, H, W), dtype=np.float32)
    _check(lib().orc_corr_f32(_ptr(L), _ptr(R), _ptr(out), B, C, H, W, D, G, nthreads), "corr_f32")
    return out if G > 1 else out.reshape(B, D, H, W)


def corr_f16(L: np.ndarray, R: np.ndarray, D: int, G: int = 1, scale_mode: int | None = None,
             nthreads: int = 0) -> np.ndarray:
    Lh, Rh = _h(L), _h(R)
    B, C, H, W = Lh.shape
    if scale_mode is None:
        scale_mode = grouped_scale_mode(True, B, C, G, H, W, D)
    out = np.empty((B, G, D, H, W), dtype=np.uint16)
    _check(lib().orc_corr_f16(_ptr(Lh), _ptr(Rh), _ptr(out), B, C, H, W, D, G, scale_mode, nthreads),
           "corr_f16")
    out = out.view(np.float16)
    return out if G > 1 else out.reshape(B, D, H, W)


def stem_ref3(vol: np.ndarray, w0, b0, w1, b1, w2, b2, nthreads: int = 0) -> np.ndarray:
    v = _h(vol)
    B, one, D, H, W = v.shape
    assert one == 1
    ws = [_h(np.asarray(x, dtype=np.float16)) for x in (w0, b0, w1, b1, w2, b2)]
    out = np.empty_like(v)
    _check(lib().orc_stem_ref3(_ptr(v), _ptr(out), *[_ptr(x) for x in ws], B, D, H, W, nthreads),
           "stem_ref3")
    return out.view(np.float16)


def stem(vol: np.ndarray, w: np.ndarray, b: np.ndarray, act: int = ACT_RELU, acc_mode: int = ACC_F64,
         batches: tuple[int, int] | None = None, rows: tuple[int, int] | None = None,
         out: np.ndarray | None = None, nthreads: int = 0) -> np.ndarray:
    v = _h(vol)
    B, Cin, D, H, W = v.shape
    wh, bh = _h(np.asarray(w, dtype=np.float16)), _h(np.asarray(b, dtype=np.float16))
    Cout = bh.shape[0]
    assert wh.size == Cout * Cin * 27
    b0, b1 = batches or (0, B)
    h0, h1 = rows or (0, H)
    if out is None:
        out = np.zeros((B, Cout, D, H, W), dtype=np.uint16)
    out = _h(out)
    _check(lib().orc_stem(_ptr(v), _ptr(wh), _ptr(bh), _ptr(out), B, Cin, Cout, D, H, W, act, acc_mode,
                          b0, b1, h0, h1, nthreads), "stem")
    return out.view(np.float16)


def corr_stem(L: np.ndarray, R: np.ndarray, w: np.ndarray, b: np.ndarray, D: int, G: int,
              act: int = ACT_RELU, scale_mode: int | None = None, acc_mode: int = ACC_F64,
              batches: tuple[int, int] | None = None, rows: tuple[int, int] | None = None,
              out: np.ndarray | None = None, nthreads: int = 0) -> np.ndarray:
    Lh, Rh = _h(L), _h(R)
    B, C, H, W = Lh.shape
    wh, bh = _h(np.asarray(w, dtype=np.float16)), _h(np.asarray(b, dtype=np.float16))
    Cout = bh.shape[0]
    assert wh.size == Cout * G * 27
    if scale_mode is None:
        scale_mode = grouped_scale_mode(True, B, C, G, H, W, D)
    b0, b1 = batches or (0, B)
    h0, h1 = rows or (0, H)
    if out is None:
        out = np.zeros((B, Cout, D, H, W), dtype=np.uint16)
    out = _h(out)
    _check(lib().orc_corr_stem(_ptr(Lh), _ptr(Rh), _ptr(wh), _ptr(bh), _ptr(out), B, C, G, H, W, D, Cout,
                               act, scale_mode, acc_mode, b0, b1, h0, h1, nthreads), "corr_stem")
    return out.view(np.float16)


def fold_bn(w: np.ndarray, scale: np.ndarray, bias: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    w = np.ascontiguousarray(w, dtype=np.float32)
    scale = np.ascontiguousarray(scale, dtype=np.float32)
    bias = np.ascontiguousarray(bias, dtype=np.float32)
    cout = w.shape[0]
    k = w.size // cout
    w16 = np.empty(w.shape, dtype=np.uint16)
    b16 = np.empty((cout,), dtype=np.uint16)
    lib().orc_fold_bn(_ptr(w), _ptr(scale), _ptr(bias), cout, k, _ptr(w16), _ptr(b16))
    return w16.view(np.float16), b16.view(np.float16)


def nv12_decode(nv12: np.ndarray, H_OUT: int, W_OUT: int, out_f16: bool = True, nthreads: int = 0) -> np.ndarray:
    """NV12 [B, H_IN * 3 / 2, W_IN] uint8 -> [B, 3, H_OUT, W_OUT] fp16 (or fp32)."""
    a = np.ascontiguousarray(nv12, dtype=np.uint8)
    if a.ndim == 2:
        a = a[None]
    B, H_NV12, W_IN = a.shape
    H_IN = H_NV12 * 2 // 3
    out = np.empty((B, 3, H_OUT, W_OUT), dtype=np.uint16 if out_f16 else np.float32)
    _check(lib().orc_nv12_decode(_ptr(a), B, H_IN, W_IN, H_OUT, W_OUT, int(out_f16), _ptr(out), nthreads),
           "nv12_decode")
    return out.view(np.float16) if out_f16 else out


def disparity_regression(cost: np.ndarray, mode: int = 0, out_f16: bool = False, nthreads: int = 0) -> np.ndarray:
    """cost [B, D, H, W] (or [B, 1, D, H, W]) fp16/fp32 -> disparity [B, 1, H, W]:
    sum_d d * softmax_d(s * cost), s = +1 (mode 0) or -1 (mode 1), in double,
    rounded once to fp32 (or fp16).  No reference counterpart exists; the
    formula is the specification."""
    a = np.ascontiguousarray(cost)
    if a.ndim == 5:
        assert a.shape[1] == 1
        a = a[:, 0]
    if a.dtype == np.float16:
        in_f16, a = 1, a.view(np.uint16)
    else:
        in_f16, a = 0, np.ascontiguousarray(a, dtype=np.float32)
    B, D, H, W = a.shape
    out = np.empty((B, 1, H, W), dtype=np.uint16 if out_f16 else np.float32)
    _check(lib().orc_disparity_regression(_ptr(a), in_f16, B, D, H, W, mode, int(out_f16), _ptr(out), nthreads),
           "disparity_regression")
    return out.view(np.float16) if out_f16 else out
