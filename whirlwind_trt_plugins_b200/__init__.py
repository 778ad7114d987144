"""B200-native stereo cost-volume front end (CorrVolume -> CostStem3D).

Python host side over the C ABI of ``libww_trt_plugins.so``
(``include/ww_trt_plugins.h``).  torch supplies device memory and streams;
every computation runs in the library's sm_100a kernels.  There is no CPU
fallback: importing this package fails loudly when the library is missing,
and every call raises ``WWError`` when the library rejects it.

Operators (reference interfaces in parentheses, paths relative to the
reference project):

* ``corr_volume(left, right, max_disp, num_groups=1)``  -- CorrVolume
  (``src/plugins/corr_volume/corr_volume_kernel.hpp:17-27``)
* ``cost_stem3d_ref3(vol, w0, b0, w1, b1, w2, b2)``     -- CostStem3D 7-input form
  (``src/plugins/cost_stem_3d/cost_stem_3d_kernel.hpp:17-30``)
* ``corr_cost_stem3d_ref3(left, right, w0..b2, max_disp)`` -- CorrVolume (G = 1)
  fused with the reference CostStem3D, bit-identical to the pair
* ``cost_stem3d(vol, w, b, act)``                      -- generalised 3-input stem
* ``corr_cost_stem3d(left, right, w, b, max_disp, num_groups, act)`` -- fused op
* ``corr_cost_stem3d_band(...)``                       -- row-band form for sharding
* ``corr_cost_stem3d_multi(...)``                      -- several devices from one thread
  (batch split, or row bands with the halo rows copied between devices)
* ``nv12_decode(nv12, out_h, out_w, dtype)``           -- Nv12Decode
  (``src/plugins/nv12_decode/nv12_decode_kernel.hpp:20-28``)
* ``disparity_regression(cost, mode, dtype)``          -- soft-argmax / soft-argmin
  after the 3-D aggregation (no reference counterpart; specified by its formula)

The plugin-level classes mirroring the reference's IPluginV3 plugins live in
``whirlwind_trt_plugins_b200.plugins``; row-band sharding over several GPUs in
``whirlwind_trt_plugins_b200.shard``.
"""
from __future__ import annotations

import ctypes
import os

__all__ = [
    "LIB_PATH", "WWError", "lib", "corr_volume", "cost_stem3d_ref3", "corr_cost_stem3d_ref3", "cost_stem3d",
    "corr_cost_stem3d", "corr_cost_stem3d_band", "nv12_decode", "disparity_regression", "fold_bn", "device_error",
    "clear_device_error", "ACT_RELU", "ACT_RELU6", "DTYPE_FLOAT", "DTYPE_HALF", "DISP_SOFTARGMAX", "DISP_SOFTARGMIN",
    "MULTI_BATCH", "MULTI_ROWS", "multi_split", "corr_cost_stem3d_multi", "CORR_ENGINE_TENSOR",
    "CORR_ENGINE_CUDA_CORES", "set_fused_corr_engine", "fused_corr_engine",
]

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libww_trt_plugins.so")

DTYPE_FLOAT = 0
DTYPE_HALF = 1
ACT_RELU = 0
ACT_RELU6 = 1
DISP_SOFTARGMAX = 0
DISP_SOFTARGMIN = 1
MULTI_BATCH = 0
MULTI_ROWS = 1
CORR_ENGINE_TENSOR = 0
CORR_ENGINE_CUDA_CORES = 1

STATUS = {
    0: "success", 1: "CUDA launch or runtime call failed", 2: "invalid tensor shape",
    3: "unsupported data type", 4: "null pointer", 5: "request outside the supported limits",
    6: "pointer not aligned as required", 7: "no usable sm_100 device",
}


class WWError(RuntimeError):
    def __init__(self, fn: str, status: int):
        super().__init__(f"{fn} failed: status {status} ({STATUS.get(status, 'unknown')})")
        self.status = status


def _load() -> ctypes.CDLL:
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `python whirlwind_trt_plugins_b200/build.py` "
            "(nvcc, sm_100a). There is no CPU fallback.")
    L = ctypes.CDLL(LIB_PATH)
    p, i, f = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
    L.ww_status_string.restype = ctypes.c_char_p
    L.ww_status_string.argtypes = [i]
    L.ww_abi_version.restype = i
    L.ww_corr_volume.argtypes = [p, p, p] + [i] * 7 + [p]
    L.ww_cost_stem3d_ref3.argtypes = [p] * 8 + [i] * 4 + [p]
    L.ww_corr_cost_stem3d_ref3.argtypes = [p] * 9 + [i] * 5 + [p]
    L.ww_cost_stem3d.argtypes = [p, p, p, p] + [i] * 7 + [p]
    L.ww_corr_cost_stem3d.argtypes = [p, p, p, p, p] + [i] * 8 + [p]
    L.ww_corr_cost_stem3d_band.argtypes = [p, p, p, p, p] + [i] * 12 + [p]
    L.ww_nv12_decode.argtypes = [p, p] + [i] * 6 + [p]
    L.ww_disparity_regression.argtypes = [p, p] + [i] * 7 + [p]
    L.ww_fold_bn_f16.argtypes = [p, p, p, i, i, p, p]
    L.ww_corr_cost_stem3d_multi.argtypes = [i, p, i, p, p, p, p, p] + [i] * 8 + [p]
    L.ww_multi_split.argtypes = [i, i, i] + [ctypes.POINTER(ctypes.c_int)] * 4
    L.ww_multi_inject_copy_failure.argtypes = [i]
    L.ww_device_error.argtypes = [ctypes.POINTER(ctypes.c_int)]
    L.ww_clear_device_error.argtypes = []
    L.ww_set_fused_corr_engine.argtypes = [i]
    L.ww_selftest_int_division.argtypes = [i, ctypes.POINTER(ctypes.c_ulonglong)]
    L.ww_get_fused_corr_engine.argtypes = []
    del f
    return L


_lib = _load()


def lib() -> ctypes.CDLL:
    return _lib


def _check(fn: str, status: int) -> None:
    if status != 0:
        raise WWError(fn, status)


def _torch():
    import torch
    return torch


def _stream_ptr(stream) -> int | None:
    torch = _torch()
    if stream is None:
        stream = torch.cuda.current_stream()
    return stream.cuda_stream if hasattr(stream, "cuda_stream") else int(stream)


def _dev(t, name: str, dtype=None):
    torch = _torch()
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise TypeError(f"{name} must be a CUDA tensor")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    if dtype is not None and t.dtype != dtype:
        raise TypeError(f"{name} must be {dtype}, got {t.dtype}")
    return t


def _out(out, shape, dtype, device, name: str = "out"):
    """The output tensor of a call: a new one, or the caller's `out` after
    checking that it is a contiguous CUDA tensor of exactly `shape` and
    `dtype` (a smaller one would let the kernel write past its end)."""
    torch = _torch()
    shape = tuple(int(s) for s in shape)
    if out is None:
        return torch.empty(shape, dtype=dtype, device=device)
    _dev(out, name, dtype)
    if tuple(out.shape) != shape:
        raise ValueError(f"{name} must have shape {shape}, got {tuple(out.shape)}")
    return out


def corr_volume(left, right, max_disp: int, num_groups: int = 1, out=None, stream=None):
    """Group-wise correlation volume.

    left, right: [B, C, H, W] fp16 or fp32 CUDA tensors.  Returns
    [B, max_disp, H, W] for num_groups == 1 (the reference CorrVolume output),
    else [B, num_groups, max_disp, H, W]."""
    torch = _torch()
    _dev(left, "left")
    _dev(right, "right", left.dtype)
    if left.shape != right.shape or left.dim() != 4:
        raise ValueError("left/right must both be [B, C, H, W]")
    dt = {torch.float16: DTYPE_HALF, torch.float32: DTYPE_FLOAT}.get(left.dtype)
    if dt is None:
        raise TypeError("corr_volume supports fp16 and fp32")
    B, C, H, W = left.shape
    shape = (B, max_disp, H, W) if num_groups == 1 else (B, num_groups, max_disp, H, W)
    out = _out(out, shape, left.dtype, left.device)
    _check("ww_corr_volume", _lib.ww_corr_volume(left.data_ptr(), right.data_ptr(), out.data_ptr(), dt,
                                                 B, C, H, W, max_disp, num_groups, _stream_ptr(stream)))
    return out


def cost_stem3d_ref3(vol, w0, b0, w1, b1, w2, b2, out=None, stream=None):
    """The reference CostStem3D (1->4->4->1, ReLU6), every batch item.  All fp16."""
    torch = _torch()
    _dev(vol, "vol", torch.float16)
    ws = [_dev(x, n, torch.float16) for x, n in zip((w0, b0, w1, b1, w2, b2), ("w0", "b0", "w1", "b1", "w2", "b2"))]
    for x, n in zip(ws, (108, 4, 432, 4, 108, 1)):
        if x.numel() != n:
            raise ValueError("CostStem3D weight/bias has the wrong size")
    if vol.dim() != 5 or vol.shape[1] != 1:
        raise ValueError("vol must be [B, 1, D, H, W]")
    B, _, D, H, W = vol.shape
    out = _out(out, vol.shape, torch.float16, vol.device)
    _check("ww_cost_stem3d_ref3", _lib.ww_cost_stem3d_ref3(vol.data_ptr(), out.data_ptr(),
                                                           *[x.data_ptr() for x in ws], B, D, H, W,
                                                           _stream_ptr(stream)))
    return out


def corr_cost_stem3d_ref3(left, right, w0, b0, w1, b1, w2, b2, max_disp: int = 48, out=None, stream=None):
    """CorrVolume (G = 1) fused with the reference CostStem3D (1->4->4->1,
    ReLU6): bit-identical to cost_stem3d_ref3(corr_volume(left, right,
    max_disp)); left, right [B, C, H, W] fp16 -> [B, 1, max_disp, H, W] fp16."""
    torch = _torch()
    _dev(left, "left", torch.float16)
    _dev(right, "right", torch.float16)
    if left.dim() != 4 or left.shape != right.shape:
        raise ValueError("left and right must both be [B, C, H, W]")
    ws = [_dev(x, n, torch.float16) for x, n in zip((w0, b0, w1, b1, w2, b2), ("w0", "b0", "w1", "b1", "w2", "b2"))]
    for x, n in zip(ws, (108, 4, 432, 4, 108, 1)):
        if x.numel() != n:
            raise ValueError("CostStem3D weight/bias has the wrong size")
    B, C, H, W = left.shape
    out = _out(out, (B, 1, max_disp, H, W), torch.float16, left.device)
    _check("ww_corr_cost_stem3d_ref3", _lib.ww_corr_cost_stem3d_ref3(
        left.data_ptr(), right.data_ptr(), out.data_ptr(), *[x.data_ptr() for x in ws], B, C, H, W, max_disp,
        _stream_ptr(stream)))
    return out


def cost_stem3d(vol, w, b, act: int = ACT_RELU, out=None, stream=None):
    """Generalised stem: Conv3d 3x3x3 pad 1 Cin->Cout + bias + ReLU/ReLU6 on tensor cores."""
    torch = _torch()
    _dev(vol, "vol", torch.float16)
    _dev(w, "w", torch.float16)
    _dev(b, "b", torch.float16)
    if vol.dim() != 5:
        raise ValueError("vol must be [B, Cin, D, H, W]")
    B, Cin, D, H, W = vol.shape
    Cout = b.numel()
    if w.numel() != Cout * Cin * 27:
        raise ValueError("w must be [Cout, Cin, 3, 3, 3]")
    out = _out(out, (B, Cout, D, H, W), torch.float16, vol.device)
    _check("ww_cost_stem3d", _lib.ww_cost_stem3d(vol.data_ptr(), w.data_ptr(), b.data_ptr(), out.data_ptr(),
                                                 B, Cin, Cout, D, H, W, act, _stream_ptr(stream)))
    return out


def corr_cost_stem3d(left, right, w, b, max_disp: int, num_groups: int, act: int = ACT_RELU, out=None,
                     stream=None):
    """Fused group-wise correlation + stem; the volume never leaves the SM.

    left, right [B, C, H, W] fp16, w [Cout, G, 3, 3, 3] fp16, b [Cout] fp16.
    Returns [B, Cout, max_disp, H, W] fp16."""
    torch = _torch()
    for t, n in ((left, "left"), (right, "right"), (w, "w"), (b, "b")):
        _dev(t, n, torch.float16)
    if left.shape != right.shape or left.dim() != 4:
        raise ValueError("left/right must both be [B, C, H, W]")
    B, C, H, W = left.shape
    Cout = b.numel()
    if w.numel() != Cout * num_groups * 27:
        raise ValueError("w must be [Cout, num_groups, 3, 3, 3]")
    out = _out(out, (B, Cout, max_disp, H, W), torch.float16, left.device)
    _check("ww_corr_cost_stem3d", _lib.ww_corr_cost_stem3d(
        left.data_ptr(), right.data_ptr(), w.data_ptr(), b.data_ptr(), out.data_ptr(),
        B, C, num_groups, H, W, max_disp, Cout, act, _stream_ptr(stream)))
    return out


def corr_cost_stem3d_band(left_band, right_band, w, b, max_disp: int, num_groups: int, H: int,
                          in_row0: int, out_row0: int, out_rows: int, act: int = ACT_RELU, out=None,
                          stream=None):
    """Rows [out_row0, out_row0+out_rows) of the fused op from an input band
    holding image rows [in_row0, in_row0 + left_band.shape[2])."""
    torch = _torch()
    for t, n in ((left_band, "left"), (right_band, "right"), (w, "w"), (b, "b")):
        _dev(t, n, torch.float16)
    if left_band.dim() != 4 or left_band.shape != right_band.shape:
        raise ValueError("left_band/right_band must both be [B, C, in_rows, W]")
    B, C, in_rows, W = left_band.shape
    Cout = b.numel()
    if w.numel() != Cout * num_groups * 27:
        raise ValueError("w must be [Cout, num_groups, 3, 3, 3]")
    out = _out(out, (B, Cout, max_disp, out_rows, W), torch.float16, left_band.device)
    _check("ww_corr_cost_stem3d_band", _lib.ww_corr_cost_stem3d_band(
        left_band.data_ptr(), right_band.data_ptr(), w.data_ptr(), b.data_ptr(), out.data_ptr(),
        B, C, num_groups, H, W, max_disp, Cout, act, in_row0, in_rows, out_row0, out_rows,
        _stream_ptr(stream)))
    return out


def multi_split(n: int, H: int, k: int) -> tuple[int, int, int, int]:
    """Rows (r0, r1) of part k of n in an H-row image and the band (i0, i1)
    it holds (one halo row each side, clipped): ww_multi_split."""
    v = [ctypes.c_int(0) for _ in range(4)]
    _check("ww_multi_split", _lib.ww_multi_split(n, H, k, *[ctypes.byref(x) for x in v]))
    return tuple(x.value for x in v)


def corr_cost_stem3d_multi(lefts, rights, ws, bs, max_disp: int, num_groups: int, mode: int = MULTI_BATCH,
                           act: int = ACT_RELU, H: int | None = None, outs=None, streams=None):
    """The fused op over several parts (each a CUDA tensor set on its own
    device; parts may share a device) through ww_corr_cost_stem3d_multi.

    MULTI_BATCH: lefts[k]/rights[k] [b_k, C, H, W] hold batch items
    split_even(B, n, k); returns outs[k] [b_k, Cout, D, H, W].
    MULTI_ROWS: lefts[k]/rights[k] [B, C, i1 - i0, W] are band buffers of an
    H-row image (multi_split) with the own rows filled; the halo rows are
    copied from the neighbours by the library; returns outs[k]
    [B, Cout, D, r1 - r0, W].  streams[k]: a torch stream of part k's device
    (default: its current stream)."""
    torch = _torch()
    n = len(lefts)
    if not (len(rights) == len(ws) == len(bs) == n) or n == 0:
        raise ValueError("one left, right, w and b per part")
    if mode not in (MULTI_BATCH, MULTI_ROWS):
        raise ValueError("mode must be MULTI_BATCH or MULTI_ROWS")
    for k in range(n):
        for t, nm in ((lefts[k], "left"), (rights[k], "right"), (ws[k], "w"), (bs[k], "b")):
            _dev(t, f"{nm}[{k}]", torch.float16)
        if lefts[k].dim() != 4 or lefts[k].shape != rights[k].shape:
            raise ValueError(f"left[{k}] and right[{k}] must both be [B, C, rows, W]")
        if not (lefts[k].device == rights[k].device == ws[k].device == bs[k].device):
            raise ValueError(f"part {k}: left, right, w and b must be on one device")
    C, W = lefts[0].shape[1], lefts[0].shape[3]
    Cout = bs[0].numel()
    if any(t.numel() != Cout * num_groups * 27 for t in ws):
        raise ValueError("w must be [Cout, num_groups, 3, 3, 3]")
    shapes = []
    if mode == MULTI_BATCH:
        H = lefts[0].shape[2]
        B = sum(t.shape[0] for t in lefts)
        for k in range(n):
            base, extra = divmod(B, n)
            bk = base + (1 if k < extra else 0)
            if lefts[k].shape != (bk, C, H, W):
                raise ValueError(f"part {k} must hold {bk} of the {B} pairs: [{bk}, {C}, {H}, {W}]")
            shapes.append((bk, Cout, max_disp, H, W))
    else:
        if H is None:
            raise ValueError("MULTI_ROWS needs the image height H")
        B = lefts[0].shape[0]
        for k in range(n):
            r0, r1, i0, i1 = multi_split(n, H, k)
            if lefts[k].shape != (B, C, i1 - i0, W):
                raise ValueError(f"part {k} must hold rows [{i0}, {i1}): [{B}, {C}, {i1 - i0}, {W}]")
            shapes.append((B, Cout, max_disp, r1 - r0, W))
    if outs is None:
        outs = [None] * n
    outs = [_out(outs[k], shapes[k], torch.float16, lefts[k].device, f"out[{k}]") for k in range(n)]
    if streams is None:
        streams = [torch.cuda.current_stream(t.device) for t in lefts]
    P = ctypes.c_void_p * n
    devs = (ctypes.c_int * n)(*[t.device.index for t in lefts])
    sp = P(*[s.cuda_stream if hasattr(s, "cuda_stream") else int(s) for s in streams])
    _check("ww_corr_cost_stem3d_multi", _lib.ww_corr_cost_stem3d_multi(
        n, devs, mode, P(*[t.data_ptr() for t in lefts]), P(*[t.data_ptr() for t in rights]),
        P(*[t.data_ptr() for t in ws]), P(*[t.data_ptr() for t in bs]), P(*[t.data_ptr() for t in outs]),
        B, C, num_groups, H, W, max_disp, Cout, act, sp))
    return outs


def nv12_decode(nv12, out_h: int = 224, out_w: int = 288, dtype=None, out=None, stream=None):
    """NV12 [B, H_IN * 3 / 2, W_IN] (uint8 or int8 bytes, or one [H*3/2, W]
    image) -> planar RGB [B, 3, out_h, out_w] in [-1, 1], fp16 (default) or
    fp32: bilinear resize (align_corners = False, clamped), full-range
    BT.601.  Every batch item is decoded."""
    torch = _torch()
    if not isinstance(nv12, torch.Tensor) or not nv12.is_cuda:
        raise TypeError("nv12 must be a CUDA tensor")
    if nv12.dtype not in (torch.uint8, torch.int8):
        raise TypeError("nv12 must hold uint8 (or int8) bytes")
    if not nv12.is_contiguous():
        raise ValueError("nv12 must be contiguous")
    x = nv12 if nv12.dim() == 3 else nv12.unsqueeze(0)
    if x.dim() != 3 or x.shape[1] % 3 != 0:
        raise ValueError("nv12 must be [B, H_IN * 3 / 2, W_IN]")
    B, H_NV12, W_IN = x.shape
    dtype = dtype or torch.float16
    dt = {torch.float16: DTYPE_HALF, torch.float32: DTYPE_FLOAT}.get(dtype)
    if dt is None:
        raise TypeError("output dtype must be float16 or float32")
    out = _out(out, (B, 3, out_h, out_w), dtype, x.device)
    _check("ww_nv12_decode", _lib.ww_nv12_decode(x.data_ptr(), out.data_ptr(), dt, B, H_NV12 * 2 // 3, W_IN,
                                                 out_h, out_w, _stream_ptr(stream)))
    return out


def disparity_regression(cost, mode: int = DISP_SOFTARGMAX, dtype=None, out=None, stream=None):
    """cost [B, D, H, W] or [B, 1, D, H, W] (fp16 or fp32) -> disparity
    [B, 1, H, W] = sum_d d * softmax_d(s * cost), s = +1 (DISP_SOFTARGMAX,
    cost is a similarity) or -1 (DISP_SOFTARGMIN, cost is a matching cost);
    fp32 arithmetic, output dtype = input dtype unless `dtype` is given."""
    torch = _torch()
    _dev(cost, "cost")
    dts = {torch.float16: DTYPE_HALF, torch.float32: DTYPE_FLOAT}
    if cost.dtype not in dts:
        raise TypeError("cost must be float16 or float32")
    if cost.dim() == 5 and cost.shape[1] == 1:
        B, _, D, H, W = cost.shape
    elif cost.dim() == 4:
        B, D, H, W = cost.shape
    else:
        raise ValueError("cost must be [B, D, H, W] or [B, 1, D, H, W]")
    if mode not in (DISP_SOFTARGMAX, DISP_SOFTARGMIN):
        raise ValueError("mode must be DISP_SOFTARGMAX or DISP_SOFTARGMIN")
    dtype = dtype or cost.dtype
    if dtype not in dts:
        raise TypeError("output dtype must be float16 or float32")
    out = _out(out, (B, 1, H, W), dtype, cost.device)
    _check("ww_disparity_regression", _lib.ww_disparity_regression(
        cost.data_ptr(), out.data_ptr(), dts[cost.dtype], dts[dtype], B, D, H, W, mode, _stream_ptr(stream)))
    return out


def fold_bn(w, scale, bias):
    """Host BatchNorm fold (numpy): fp16(w * scale[o]) and fp16(bias)."""
    import numpy as np
    w = np.ascontiguousarray(w, dtype=np.float32)
    scale = np.ascontiguousarray(scale, dtype=np.float32)
    bias = np.ascontiguousarray(bias, dtype=np.float32)
    cout = w.shape[0]
    k = w.size // cout
    w16 = np.empty(w.shape, dtype=np.uint16)
    b16 = np.empty((cout,), dtype=np.uint16)
    _check("ww_fold_bn_f16", _lib.ww_fold_bn_f16(w.ctypes.data, scale.ctypes.data, bias.ctypes.data, cout, k,
                                                 w16.ctypes.data, b16.ctypes.data))
    return w16.view(np.float16), b16.view(np.float16)


def set_fused_corr_engine(engine: int) -> int:
    """Select the fused op's correlation engine (CORR_ENGINE_TENSOR, the
    default, or CORR_ENGINE_CUDA_CORES: a channel-order fp32 fma chain whose
    volume equals corr_volume's bit for bit); returns the previous one."""
    prev = _lib.ww_set_fused_corr_engine(int(engine))
    if engine not in (CORR_ENGINE_TENSOR, CORR_ENGINE_CUDA_CORES):
        _check("ww_set_fused_corr_engine", prev)
    return prev


def fused_corr_engine() -> int:
    return _lib.ww_get_fused_corr_engine()


def device_error() -> int:
    """Error word written by bounded device-side waits (0 = none); synchronises."""
    code = ctypes.c_int(0)
    _check("ww_device_error", _lib.ww_device_error(ctypes.byref(code)))
    return code.value


def clear_device_error() -> None:
    _check("ww_clear_device_error", _lib.ww_clear_device_error())
