// ww_trt_plugins.cpp -- TensorRT (10.x, IPluginV3) front end of the B200
// library.  Compiled only where TensorRT's headers and libnvinfer exist:
//
//   g++ -std=c++17 -O2 -fPIC -shared -I<repo>/include -I<tensorrt>/include
//       -I<cuda>/include ww_trt_plugins.cpp -L<repo>/whirlwind_trt_plugins_b200
//       -lww_trt_plugins -L<tensorrt>/lib -lnvinfer -o libww_trt_shim.so
//
// It registers the creators the reference registers
// (src/register_plugins.cpp:15-18, the stereo path and the camera decode)
// under the same names and version -- "CorrVolume" v"1" with field max_disp
// (default 48), "CostStem3D" v"1" with no required field, "Nv12Decode" v"1"
// with fields out_h / out_w (224 / 288) -- plus the fused "CorrCostStem3D" and
// "DisparityRegression" (field mode), which have no reference counterpart.  Every method is
// a thin forwarder to the ww_plugin_* functions of the C ABI (plugin_core.cpp),
// which carry the logic of the reference's IPluginV3 methods
// (src/plugins/corr_volume/corr_volume.cpp:23-139,
// src/plugins/cost_stem_3d/cost_stem_3d.cpp:14-97,
// src/plugins/nv12_decode/nv12_decode.cpp:16-146).  One plugin class serves
// every op; the op kind selects the forwarding target.
#include <NvInferRuntime.h>
#include <NvInferRuntimePlugin.h>
#include <NvInferPlugin.h>

#include <array>
#include <cstring>
#include <new>
#include <string>
#include <vector>

#include "ww_trt_plugins.h"

namespace ww_trt {

using namespace nvinfer1;

enum class Op { kCorrVolume, kCostStem3D, kCorrCostStem3D, kNv12Decode, kDisparityRegression };

// Integer fields an op carries; every op stores all three, serialises its own.
struct Fields {
    int32_t max_disp = 48;
    int32_t num_groups = 1;
    int32_t act = WW_ACT_RELU;
    int32_t out_h = 224;
    int32_t out_w = 288;
    int32_t mode = WW_DISP_SOFTARGMAX;
};

constexpr char const* kVersion = "1";

char const* op_name(Op op) noexcept
{
    switch (op) {
        case Op::kCorrVolume: return "CorrVolume";
        case Op::kCostStem3D: return "CostStem3D";
        case Op::kCorrCostStem3D: return "CorrCostStem3D";
        case Op::kNv12Decode: return "Nv12Decode";
        case Op::kDisparityRegression: return "DisparityRegression";
    }
    return "";
}

// Field names an op accepts at creation and writes at serialisation.
std::vector<char const*> op_fields(Op op)
{
    switch (op) {
        case Op::kCorrVolume: return {"max_disp", "num_groups"};
        case Op::kCostStem3D: return {"act"};
        case Op::kCorrCostStem3D: return {"max_disp", "num_groups", "act"};
        case Op::kNv12Decode: return {"out_h", "out_w"};
        case Op::kDisparityRegression: return {"mode"};
    }
    return {};
}

int32_t* field_slot(Fields& f, char const* name) noexcept
{
    if (std::strcmp(name, "max_disp") == 0) return &f.max_disp;
    if (std::strcmp(name, "num_groups") == 0) return &f.num_groups;
    if (std::strcmp(name, "act") == 0) return &f.act;
    if (std::strcmp(name, "out_h") == 0) return &f.out_h;
    if (std::strcmp(name, "out_w") == 0) return &f.out_w;
    if (std::strcmp(name, "mode") == 0) return &f.mode;
    return nullptr;
}

ww_tensor_desc_t to_ww(PluginTensorDesc const& d) noexcept
{
    ww_tensor_desc_t w{};
    w.nb_dims = d.dims.nbDims;
    for (int i = 0; i < d.dims.nbDims && i < 8; ++i) w.dims[i] = d.dims.d[i];
    w.dtype = static_cast<int32_t>(d.type);     // kFLOAT = 0, kHALF = 1
    w.format = static_cast<int32_t>(d.format);  // kLINEAR = 0
    return w;
}

class WwPlugin final : public IPluginV3,
                       public IPluginV3OneCore,
                       public IPluginV3OneBuild,
                       public IPluginV3OneRuntime {
public:
    WwPlugin(Op op, Fields f, std::string ns, int nb_inputs = 0)
        : mOp(op), mFields(f), mNamespace(std::move(ns)), mNbInputs(nb_inputs)
    {
    }

    // IPluginV3
    IPluginCapability* getCapabilityInterface(PluginCapabilityType type) noexcept override
    {
        if (type == PluginCapabilityType::kCORE) return static_cast<IPluginV3OneCore*>(this);
        if (type == PluginCapabilityType::kBUILD) return static_cast<IPluginV3OneBuild*>(this);
        if (type == PluginCapabilityType::kRUNTIME) return static_cast<IPluginV3OneRuntime*>(this);
        return nullptr;
    }
    IPluginV3* clone() noexcept override
    {
        return new (std::nothrow) WwPlugin(mOp, mFields, mNamespace, mNbInputs);
    }

    // IPluginV3OneCore
    AsciiChar const* getPluginName() const noexcept override { return op_name(mOp); }
    AsciiChar const* getPluginVersion() const noexcept override { return kVersion; }
    AsciiChar const* getPluginNamespace() const noexcept override { return mNamespace.c_str(); }

    // IPluginV3OneBuild
    int32_t getNbOutputs() const noexcept override { return 1; }

    int32_t configurePlugin(DynamicPluginTensorDesc const*, int32_t nbInputs, DynamicPluginTensorDesc const*,
                            int32_t) noexcept override
    {
        mNbInputs = nbInputs;
        return 0;
    }

    int32_t getOutputDataTypes(DataType* out, int32_t nbOutputs, DataType const* in,
                               int32_t nbInputs) const noexcept override
    {
        if (nbOutputs < 1 || nbInputs < 1) return 1;
        // Nv12Decode declares fp32 and lets the format choice pick fp16 or
        // fp32 (nv12_decode.cpp:26-39); the others follow input 0.
        out[0] = mOp == Op::kNv12Decode ? DataType::kFLOAT : in[0];
        return 0;
    }

    int32_t getOutputShapes(DimsExprs const* in, int32_t nbInputs, DimsExprs const*, int32_t, DimsExprs* out,
                            int32_t nbOutputs, IExprBuilder& eb) noexcept override
    {
        if (nbOutputs != 1) return 1;
        switch (mOp) {
            case Op::kCorrVolume:  // [B, D, H, W] or [B, G, D, H, W]
                if (nbInputs != 2 || in[0].nbDims != 4) return 1;
                if (mFields.num_groups <= 1) {
                    out[0].nbDims = 4;
                    out[0].d[0] = in[0].d[0];
                    out[0].d[1] = eb.constant(mFields.max_disp);
                    out[0].d[2] = in[0].d[2];
                    out[0].d[3] = in[0].d[3];
                } else {
                    out[0].nbDims = 5;
                    out[0].d[0] = in[0].d[0];
                    out[0].d[1] = eb.constant(mFields.num_groups);
                    out[0].d[2] = eb.constant(mFields.max_disp);
                    out[0].d[3] = in[0].d[2];
                    out[0].d[4] = in[0].d[3];
                }
                return 0;
            case Op::kCostStem3D:  // 7 inputs: shape of input 0; 3 inputs: Cout from w
                if (nbInputs == 7) {
                    out[0] = in[0];
                    return 0;
                }
                if (nbInputs != 3 || in[0].nbDims != 5 || in[1].nbDims != 5) return 1;
                out[0] = in[0];
                out[0].d[1] = in[1].d[0];
                return 0;
            case Op::kNv12Decode:  // [B, H * 3 / 2, W] -> [B, 3, out_h, out_w]
                if (nbInputs != 1 || in[0].nbDims != 3) return 1;
                out[0].nbDims = 4;
                out[0].d[0] = in[0].d[0];
                out[0].d[1] = eb.constant(3);
                out[0].d[2] = eb.constant(mFields.out_h);
                out[0].d[3] = eb.constant(mFields.out_w);
                return 0;
            case Op::kDisparityRegression:  // [B, D, H, W] or [B, 1, D, H, W] -> [B, 1, H, W]
                if (nbInputs != 1 || (in[0].nbDims != 4 && in[0].nbDims != 5)) return 1;
                out[0].nbDims = 4;
                out[0].d[0] = in[0].d[0];
                out[0].d[1] = eb.constant(1);
                out[0].d[2] = in[0].d[in[0].nbDims - 2];
                out[0].d[3] = in[0].d[in[0].nbDims - 1];
                return 0;
            case Op::kCorrCostStem3D:  // [B, Cout, D, H, W]; 8 inputs (3-stage stem): Cout = 1
                if ((nbInputs != 4 && nbInputs != 8) || in[0].nbDims != 4) return 1;
                if (nbInputs == 4 && in[2].nbDims != 5) return 1;
                out[0].nbDims = 5;
                out[0].d[0] = in[0].d[0];
                out[0].d[1] = nbInputs == 8 ? eb.constant(1) : in[2].d[0];
                out[0].d[2] = eb.constant(mFields.max_disp);
                out[0].d[3] = in[0].d[2];
                out[0].d[4] = in[0].d[3];
                return 0;
        }
        return 1;
    }

    bool supportsFormatCombination(int32_t pos, DynamicPluginTensorDesc const* inOut, int32_t nbInputs,
                                   int32_t nbOutputs) noexcept override
    {
        const int n = nbInputs + nbOutputs;
        if (n <= 0 || n > 9) return false;  // up to 8 inputs + 1 output
        std::array<ww_tensor_desc_t, 9> d{};
        for (int i = 0; i < n; ++i) d[i] = to_ww(inOut[i].desc);
        switch (mOp) {
            case Op::kCorrVolume:
                return ww_plugin_corr_volume_supports_format(pos, d.data(), nbInputs, nbOutputs) != 0;
            case Op::kCostStem3D:
                return ww_plugin_cost_stem3d_supports_format(pos, d.data(), nbInputs, nbOutputs) != 0;
            case Op::kCorrCostStem3D:
                return ww_plugin_corr_cost_stem3d_supports_format(pos, d.data(), nbInputs, nbOutputs) != 0;
            case Op::kNv12Decode:
                return ww_plugin_nv12_decode_supports_format(pos, d.data(), nbInputs, nbOutputs) != 0;
            case Op::kDisparityRegression:
                return ww_plugin_disparity_regression_supports_format(pos, d.data(), nbInputs, nbOutputs) != 0;
        }
        return false;
    }

    size_t getWorkspaceSize(DynamicPluginTensorDesc const*, int32_t, DynamicPluginTensorDesc const*,
                            int32_t) const noexcept override
    {
        return 0;  // no kernel of this library uses scratch memory
    }

    // IPluginV3OneRuntime
    int32_t onShapeChange(PluginTensorDesc const*, int32_t nbInputs, PluginTensorDesc const*,
                          int32_t) noexcept override
    {
        mNbInputs = nbInputs;
        return 0;
    }

    int32_t enqueue(PluginTensorDesc const* inDesc, PluginTensorDesc const* outDesc, void const* const* inputs,
                    void* const* outputs, void*, cudaStream_t stream) noexcept override
    {
        // Descriptors of the inputs: 2 (CorrVolume), 7 or 3 (CostStem3D), 4 or 8 (fused).
        std::array<ww_tensor_desc_t, 8> d{};
        const int nin = mNbInputs;
        if (nin < 1 || nin > 8) return 1;
        for (int i = 0; i < nin; ++i) d[i] = to_ww(inDesc[i]);
        switch (mOp) {
            case Op::kCorrVolume:
                return ww_plugin_corr_volume_enqueue(mFields.max_disp, mFields.num_groups, d.data(), inputs,
                                                     outputs, stream);
            case Op::kCostStem3D:
                return ww_plugin_cost_stem3d_enqueue(nin, mFields.act, d.data(), inputs, outputs, stream);
            case Op::kCorrCostStem3D:
                return ww_plugin_corr_cost_stem3d_enqueue(nin, mFields.max_disp, mFields.num_groups, mFields.act,
                                                          d.data(), inputs, outputs, stream);
            case Op::kNv12Decode: {
                if (outDesc == nullptr) return 1;
                const ww_tensor_desc_t od = to_ww(outDesc[0]);
                return ww_plugin_nv12_decode_enqueue(mFields.out_h, mFields.out_w, d.data(), &od, inputs, outputs,
                                                     stream);
            }
            case Op::kDisparityRegression: {
                if (outDesc == nullptr) return 1;
                const ww_tensor_desc_t od = to_ww(outDesc[0]);
                return ww_plugin_disparity_regression_enqueue(mFields.mode, d.data(), &od, inputs, outputs, stream);
            }
        }
        return 1;
    }

    IPluginV3* attachToContext(IPluginResourceContext*) noexcept override { return clone(); }

    PluginFieldCollection const* getFieldsToSerialize() noexcept override
    {
        mSerial.clear();
        for (char const* name : op_fields(mOp)) {
            int32_t* v = field_slot(mFields, name);
            // The reference's CostStem3D serialises nothing; keep that unless
            // the extension field differs from its default.
            if (mOp == Op::kCostStem3D && *v == WW_ACT_RELU) continue;
            mSerial.emplace_back(name, v, PluginFieldType::kINT32, 1);
        }
        mSerialFc.nbFields = static_cast<int32_t>(mSerial.size());
        mSerialFc.fields = mSerial.data();
        return &mSerialFc;
    }

private:
    Op mOp;
    Fields mFields;
    std::string mNamespace;
    int mNbInputs;  // from configurePlugin / onShapeChange (CostStem3D takes 7 or 3)
    std::vector<PluginField> mSerial;
    PluginFieldCollection mSerialFc{};
};

class WwCreator : public IPluginCreatorV3One {
public:
    explicit WwCreator(Op op) : mOp(op)
    {
        for (char const* name : op_fields(op)) mFieldList.emplace_back(name, nullptr, PluginFieldType::kINT32, 1);
        mFc.nbFields = static_cast<int32_t>(mFieldList.size());
        mFc.fields = mFieldList.data();
    }

    IPluginV3* createPlugin(AsciiChar const*, PluginFieldCollection const* fc, TensorRTPhase) noexcept override
    {
        Fields f;
        if (fc != nullptr && fc->fields != nullptr) {
            // First field of a name with data wins; absent or empty keeps the default.
            std::vector<char const*> names(fc->nbFields);
            std::vector<int32_t const*> values(fc->nbFields);
            for (int i = 0; i < fc->nbFields; ++i) {
                names[i] = fc->fields[i].name;
                values[i] = fc->fields[i].type == PluginFieldType::kINT32
                                ? static_cast<int32_t const*>(fc->fields[i].data)
                                : nullptr;
            }
            for (char const* name : op_fields(mOp)) {
                int32_t* slot = field_slot(f, name);
                *slot = ww_plugin_get_int_field(fc->nbFields, names.data(), values.data(), name, *slot);
            }
        }
        auto* p = new (std::nothrow) WwPlugin(mOp, f, mNamespace);
        return p;
    }

    PluginFieldCollection const* getFieldNames() noexcept override { return &mFc; }
    AsciiChar const* getPluginName() const noexcept override { return op_name(mOp); }
    AsciiChar const* getPluginVersion() const noexcept override { return kVersion; }
    AsciiChar const* getPluginNamespace() const noexcept override { return mNamespace.c_str(); }
    void setPluginNamespace(char const* ns) noexcept { mNamespace = ns ? ns : ""; }

private:
    Op mOp;
    std::string mNamespace;
    std::vector<PluginField> mFieldList;
    PluginFieldCollection mFc{};
};

struct CorrVolumeCreator final : WwCreator {
    CorrVolumeCreator() : WwCreator(Op::kCorrVolume) {}
};
struct CostStem3DCreator final : WwCreator {
    CostStem3DCreator() : WwCreator(Op::kCostStem3D) {}
};
struct CorrCostStem3DCreator final : WwCreator {
    CorrCostStem3DCreator() : WwCreator(Op::kCorrCostStem3D) {}
};
struct Nv12DecodeCreator final : WwCreator {
    Nv12DecodeCreator() : WwCreator(Op::kNv12Decode) {}
};
struct DisparityRegressionCreator final : WwCreator {
    DisparityRegressionCreator() : WwCreator(Op::kDisparityRegression) {}
};

}  // namespace ww_trt

// The registration macro pastes the creator's name into an identifier, so it
// takes unqualified names.
using ww_trt::CorrCostStem3DCreator;
using ww_trt::CorrVolumeCreator;
using ww_trt::CostStem3DCreator;
using ww_trt::DisparityRegressionCreator;
using ww_trt::Nv12DecodeCreator;

REGISTER_TENSORRT_PLUGIN(CorrVolumeCreator);
REGISTER_TENSORRT_PLUGIN(CostStem3DCreator);
REGISTER_TENSORRT_PLUGIN(CorrCostStem3DCreator);
REGISTER_TENSORRT_PLUGIN(Nv12DecodeCreator);
REGISTER_TENSORRT_PLUGIN(DisparityRegressionCreator);
