"""Plugin-level host mirror of the reference's TensorRT plugins.

The reference registers IPluginV3 plugins with TensorRT
(``src/register_plugins.cpp:15-16``).  This module gives the same objects
without TensorRT: a creator per plugin name/version that builds a plugin from
a field collection, and plugins with the IPluginV3 methods a caller uses
(``get_output_data_types``, ``get_output_shapes``,
``supports_format_combination``, ``get_fields_to_serialize``, ``clone``,
``enqueue``).  Every method forwards to the ``ww_plugin_*`` functions of the C
ABI, which the TensorRT shim (``csrc/trt/ww_trt_plugins.cpp``) forwards to as
well, so both front ends share one implementation.

Reference plugins (paths relative to the reference project):

* ``CorrVolume`` v1, field ``max_disp`` (default 48) --
  ``src/plugins/corr_volume/corr_volume.cpp:23-139``; extension field
  ``num_groups`` (default 1, the reference behaviour).
* ``CostStem3D`` v1, no fields, 7 inputs --
  ``src/plugins/cost_stem_3d/cost_stem_3d.cpp:14-97``; extension: a 3-input
  form (vol, w, b) with field ``act``.
* ``CorrCostStem3D`` v1 (extension, the fused op): fields ``max_disp``,
  ``num_groups``, ``act``.
* ``Nv12Decode`` v1, fields ``out_h`` (224), ``out_w`` (288) --
  ``src/plugins/nv12_decode/nv12_decode.cpp:16-146``.
* ``DisparityRegression`` v1 (extension, no reference counterpart): field
  ``mode`` (0 soft-argmax, 1 soft-argmin).

Descriptors are :class:`TensorDesc` (dims, dtype, format); dtypes use
TensorRT's numbering (0 = kFLOAT, 1 = kHALF, 2 = kINT8), format 0 = kLINEAR.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, field

from . import lib

__all__ = ["TensorDesc", "CorrVolumePlugin", "CostStem3DPlugin", "CorrCostStem3DPlugin", "Nv12DecodePlugin",
           "DisparityRegressionPlugin", "PluginCreator", "get_plugin_creator", "registered_creators"]

DTYPE_FLOAT = 0
DTYPE_HALF = 1
DTYPE_INT8 = 2
FORMAT_LINEAR = 0


class _Desc(ctypes.Structure):
    _fields_ = [("nb_dims", ctypes.c_int32), ("dims", ctypes.c_int64 * 8),
                ("dtype", ctypes.c_int32), ("format", ctypes.c_int32)]


@dataclass
class TensorDesc:
    dims: tuple
    dtype: int = DTYPE_HALF
    format: int = FORMAT_LINEAR

    def _c(self) -> _Desc:
        if len(self.dims) > 8:
            raise ValueError("at most 8 dimensions")
        d = _Desc()
        d.nb_dims = len(self.dims)
        for i, v in enumerate(self.dims):
            d.dims[i] = int(v)
        d.dtype, d.format = int(self.dtype), int(self.format)
        return d

    @staticmethod
    def _from_c(d: _Desc) -> "TensorDesc":
        return TensorDesc(tuple(int(d.dims[i]) for i in range(d.nb_dims)), int(d.dtype), int(d.format))

    @staticmethod
    def of(t) -> "TensorDesc":
        """Descriptor of a torch tensor (fp16 or fp32)."""
        import torch
        dt = {torch.float16: DTYPE_HALF, torch.float32: DTYPE_FLOAT, torch.int8: DTYPE_INT8,
              torch.uint8: DTYPE_INT8}.get(t.dtype, -1)
        return TensorDesc(tuple(t.shape), dt, FORMAT_LINEAR)


def _descs(ds) -> ctypes.Array:
    arr = (_Desc * max(1, len(ds)))()
    for i, d in enumerate(ds):
        arr[i] = d._c()
    return arr


def _ptrs(ts) -> ctypes.Array:
    arr = (ctypes.c_void_p * max(1, len(ts)))()
    for i, t in enumerate(ts):
        arr[i] = t.data_ptr() if hasattr(t, "data_ptr") else t
    return arr


def _stream(stream):
    if stream is None:
        import torch
        return torch.cuda.current_stream().cuda_stream
    return stream.cuda_stream if hasattr(stream, "cuda_stream") else int(stream)


class _PluginBase:
    NAME = ""
    VERSION = "1"
    NB_OUTPUTS = 1

    def __init__(self):
        self.namespace = ""

    # IPluginV3OneCore
    def get_plugin_name(self) -> str:
        return self.NAME

    def get_plugin_version(self) -> str:
        return self.VERSION

    def get_nb_outputs(self) -> int:
        return self.NB_OUTPUTS

    def clone(self):
        p = type(self)(**self.get_fields_to_serialize())
        p.namespace = self.namespace
        return p

    # IPluginV3OneBuild
    def get_output_data_types(self, input_types) -> list:
        """Output type = input 0 type (corr_volume.cpp:28-37, cost_stem_3d.cpp:19-26)."""
        if len(input_types) < 1:
            raise ValueError("at least one input")
        dt = (ctypes.c_int32 * len(input_types))(*input_types)
        out = ctypes.c_int32(-1)
        if lib().ww_plugin_corr_volume_output_dtype(len(input_types), dt, ctypes.byref(out)) != 0:
            raise ValueError("getOutputDataTypes failed")
        return [out.value]


class CorrVolumePlugin(_PluginBase):
    """``CorrVolume`` (corr_volume.cpp:23-123)."""
    NAME = "CorrVolume"

    def __init__(self, max_disp: int = 48, num_groups: int = 1):
        super().__init__()
        self.max_disp = int(max_disp)
        self.num_groups = int(num_groups)

    def get_fields_to_serialize(self) -> dict:
        f = {"max_disp": self.max_disp}
        if self.num_groups != 1:
            f["num_groups"] = self.num_groups
        return f

    def get_output_shapes(self, inputs) -> list:
        out = _Desc()
        if lib().ww_plugin_corr_volume_output_dims(self.max_disp, self.num_groups, len(inputs),
                                                   _descs(inputs), ctypes.byref(out)) != 0:
            raise ValueError("CorrVolume takes two [B, C, H, W] inputs")
        return [TensorDesc._from_c(out).dims]

    def supports_format_combination(self, pos: int, in_out, nb_inputs: int, nb_outputs: int) -> bool:
        return bool(lib().ww_plugin_corr_volume_supports_format(pos, _descs(in_out), nb_inputs, nb_outputs))

    def enqueue(self, input_desc, inputs, outputs, stream=None) -> int:
        return lib().ww_plugin_corr_volume_enqueue(self.max_disp, self.num_groups, _descs(input_desc),
                                                   _ptrs(inputs), _ptrs(outputs), ctypes.c_void_p(_stream(stream)))


class CostStem3DPlugin(_PluginBase):
    """``CostStem3D`` (cost_stem_3d.cpp:14-81): 7 inputs (reference) or 3 (extension)."""
    NAME = "CostStem3D"

    def __init__(self, act: int = 0):
        super().__init__()
        self.act = int(act)

    def get_fields_to_serialize(self) -> dict:
        # The reference serialises nothing (cost_stem_3d.cpp:75-81).
        return {"act": self.act} if self.act != 0 else {}

    def get_output_shapes(self, inputs) -> list:
        out = _Desc()
        if lib().ww_plugin_cost_stem3d_output_dims(len(inputs), _descs(inputs), ctypes.byref(out)) != 0:
            raise ValueError("CostStem3D takes 7 inputs (reference) or 3 (vol, w, b)")
        return [TensorDesc._from_c(out).dims]

    def supports_format_combination(self, pos: int, in_out, nb_inputs: int, nb_outputs: int) -> bool:
        return bool(lib().ww_plugin_cost_stem3d_supports_format(pos, _descs(in_out), nb_inputs, nb_outputs))

    def enqueue(self, input_desc, inputs, outputs, stream=None) -> int:
        return lib().ww_plugin_cost_stem3d_enqueue(len(input_desc), self.act, _descs(input_desc), _ptrs(inputs),
                                                   _ptrs(outputs), ctypes.c_void_p(_stream(stream)))


class CorrCostStem3DPlugin(_PluginBase):
    """``CorrCostStem3D`` (extension): CorrVolume fused with a G -> Cout stem
    (inputs left, right, w, b); with 8 inputs (left, right, w0, b0, w1, b1,
    w2, b2; num_groups 1) CorrVolume fused with the reference's 3-stage
    CostStem3D, bit-identical to the CorrVolume -> CostStem3D pair."""
    NAME = "CorrCostStem3D"

    def __init__(self, max_disp: int = 48, num_groups: int = 1, act: int = 0):
        super().__init__()
        self.max_disp = int(max_disp)
        self.num_groups = int(num_groups)
        self.act = int(act)

    def get_fields_to_serialize(self) -> dict:
        return {"max_disp": self.max_disp, "num_groups": self.num_groups, "act": self.act}

    def get_output_shapes(self, inputs) -> list:
        out = _Desc()
        if lib().ww_plugin_corr_cost_stem3d_output_dims(self.max_disp, self.num_groups, len(inputs),
                                                        _descs(inputs), ctypes.byref(out)) != 0:
            raise ValueError("CorrCostStem3D takes left, right [B,C,H,W], w [Cout,G,3,3,3], b [Cout] "
                             "(or left, right and the six 3-stage weights)")
        return [TensorDesc._from_c(out).dims]

    def supports_format_combination(self, pos: int, in_out, nb_inputs: int, nb_outputs: int) -> bool:
        return bool(lib().ww_plugin_corr_cost_stem3d_supports_format(pos, _descs(in_out), nb_inputs, nb_outputs))

    def enqueue(self, input_desc, inputs, outputs, stream=None) -> int:
        return lib().ww_plugin_corr_cost_stem3d_enqueue(len(input_desc), self.max_disp, self.num_groups, self.act,
                                                        _descs(input_desc), _ptrs(inputs), _ptrs(outputs),
                                                        ctypes.c_void_p(_stream(stream)))


class Nv12DecodePlugin(_PluginBase):
    """``Nv12Decode`` (nv12_decode.cpp:16-127): one INT8 input (uint8 NV12
    bytes), one fp16/fp32 output; decodes every batch item."""
    NAME = "Nv12Decode"

    def __init__(self, out_h: int = 224, out_w: int = 288):
        super().__init__()
        self.out_h = int(out_h)
        self.out_w = int(out_w)

    def get_fields_to_serialize(self) -> dict:
        return {"out_h": self.out_h, "out_w": self.out_w}

    def get_output_data_types(self, input_types) -> list:
        out = ctypes.c_int32(-1)
        if lib().ww_plugin_nv12_decode_output_dtype(len(input_types), ctypes.byref(out)) != 0:
            raise ValueError("getOutputDataTypes failed")
        return [out.value]

    def get_output_shapes(self, inputs) -> list:
        out = _Desc()
        if lib().ww_plugin_nv12_decode_output_dims(self.out_h, self.out_w, len(inputs), _descs(inputs),
                                                   ctypes.byref(out)) != 0:
            raise ValueError("Nv12Decode takes one [B, H * 3 / 2, W] input")
        return [TensorDesc._from_c(out).dims]

    def supports_format_combination(self, pos: int, in_out, nb_inputs: int, nb_outputs: int) -> bool:
        return bool(lib().ww_plugin_nv12_decode_supports_format(pos, _descs(in_out), nb_inputs, nb_outputs))

    def enqueue(self, input_desc, output_desc, inputs, outputs, stream=None) -> int:
        return lib().ww_plugin_nv12_decode_enqueue(self.out_h, self.out_w, _descs(input_desc),
                                                   _descs(output_desc), _ptrs(inputs), _ptrs(outputs),
                                                   ctypes.c_void_p(_stream(stream)))


class DisparityRegressionPlugin(_PluginBase):
    """``DisparityRegression`` (extension): cost [B, D, H, W] or [B, 1, D, H, W]
    fp16/fp32 -> disparity [B, 1, H, W] of the same dtype."""
    NAME = "DisparityRegression"

    def __init__(self, mode: int = 0):
        super().__init__()
        self.mode = int(mode)

    def get_fields_to_serialize(self) -> dict:
        return {"mode": self.mode}

    def get_output_shapes(self, inputs) -> list:
        out = _Desc()
        if lib().ww_plugin_disparity_regression_output_dims(len(inputs), _descs(inputs), ctypes.byref(out)) != 0:
            raise ValueError("DisparityRegression takes one [B, D, H, W] or [B, 1, D, H, W] input")
        return [TensorDesc._from_c(out).dims]

    def supports_format_combination(self, pos: int, in_out, nb_inputs: int, nb_outputs: int) -> bool:
        return bool(lib().ww_plugin_disparity_regression_supports_format(pos, _descs(in_out), nb_inputs,
                                                                         nb_outputs))

    def enqueue(self, input_desc, output_desc, inputs, outputs, stream=None) -> int:
        return lib().ww_plugin_disparity_regression_enqueue(self.mode, _descs(input_desc), _descs(output_desc),
                                                            _ptrs(inputs), _ptrs(outputs),
                                                            ctypes.c_void_p(_stream(stream)))


@dataclass
class PluginCreator:
    """IPluginCreatorV3One counterpart: name, version, field names, create."""
    plugin_cls: type
    field_defaults: dict = field(default_factory=dict)

    @property
    def name(self) -> str:
        return self.plugin_cls.NAME

    @property
    def version(self) -> str:
        return self.plugin_cls.VERSION

    def get_field_names(self) -> list:
        return list(self.field_defaults)

    def create_plugin(self, fields: dict | None = None):
        """Fields absent or None fall back to the defaults (plugin_fields.hpp:17-31)."""
        fields = fields or {}
        kw = {}
        for k, dflt in self.field_defaults.items():
            v = fields.get(k)
            kw[k] = dflt if v is None else int(v)
        return self.plugin_cls(**kw)


_CREATORS = {
    ("CorrVolume", "1"): PluginCreator(CorrVolumePlugin, {"max_disp": 48, "num_groups": 1}),
    ("CostStem3D", "1"): PluginCreator(CostStem3DPlugin, {"act": 0}),
    ("CorrCostStem3D", "1"): PluginCreator(CorrCostStem3DPlugin, {"max_disp": 48, "num_groups": 1, "act": 0}),
    ("Nv12Decode", "1"): PluginCreator(Nv12DecodePlugin, {"out_h": 224, "out_w": 288}),
    ("DisparityRegression", "1"): PluginCreator(DisparityRegressionPlugin, {"mode": 0}),
}


def get_plugin_creator(name: str, version: str = "1") -> PluginCreator:
    try:
        return _CREATORS[(name, version)]
    except KeyError:
        raise KeyError(f"no plugin creator {name!r} version {version!r}") from None


def registered_creators() -> list:
    return sorted(_CREATORS)
