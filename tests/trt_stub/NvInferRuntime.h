// Stand-in declarations of the TensorRT 10 plugin interface (IPluginV3 and
// its creator), written for this repository's tests: just enough of the
// public API's names and signatures for `g++ -fsyntax-only` to check the
// plugin shim (whirlwind_trt_plugins_b200/csrc/trt/ww_trt_plugins.cpp) where
// TensorRT is not installed.  Not TensorRT, and nothing links against it.
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda_runtime_api.h>

namespace nvinfer1 {

using AsciiChar = char;

enum class DataType : int32_t { kFLOAT = 0, kHALF = 1, kINT8 = 2, kINT32 = 3 };
enum class TensorFormat : int32_t { kLINEAR = 0 };

struct Dims {
    static constexpr int32_t MAX_DIMS = 8;
    int32_t nbDims;
    int64_t d[MAX_DIMS];
};

class IDimensionExpr {
public:
    virtual ~IDimensionExpr() = default;
};

struct DimsExprs {
    int32_t nbDims;
    IDimensionExpr const* d[Dims::MAX_DIMS];
};

class IExprBuilder {
public:
    virtual ~IExprBuilder() = default;
    virtual IDimensionExpr const* constant(int64_t value) noexcept = 0;
};

struct PluginTensorDesc {
    Dims dims;
    DataType type;
    TensorFormat format;
    float scale;
};

struct DynamicPluginTensorDesc {
    PluginTensorDesc desc;
    Dims min;
    Dims max;
    Dims opt;
};

enum class PluginFieldType : int32_t { kFLOAT16, kFLOAT32, kFLOAT64, kINT8, kINT16, kINT32, kCHAR, kDIMS, kUNKNOWN };

struct PluginField {
    AsciiChar const* name;
    void const* data;
    PluginFieldType type;
    int32_t length;
    PluginField(AsciiChar const* name_ = nullptr, void const* data_ = nullptr,
                PluginFieldType type_ = PluginFieldType::kUNKNOWN, int32_t length_ = 0) noexcept
        : name(name_), data(data_), type(type_), length(length_)
    {
    }
};

struct PluginFieldCollection {
    int32_t nbFields;
    PluginField const* fields;
};

enum class PluginCapabilityType : int32_t { kCORE = 0, kBUILD = 1, kRUNTIME = 2 };
enum class TensorRTPhase : int32_t { kBUILD = 0, kRUNTIME = 1 };

class IPluginResourceContext;

class IPluginCapability {
public:
    virtual ~IPluginCapability() = default;
};

class IPluginV3 : public IPluginCapability {
public:
    virtual IPluginCapability* getCapabilityInterface(PluginCapabilityType type) noexcept = 0;
    virtual IPluginV3* clone() noexcept = 0;
};

class IPluginV3OneCore : public IPluginCapability {
public:
    virtual AsciiChar const* getPluginName() const noexcept = 0;
    virtual AsciiChar const* getPluginVersion() const noexcept = 0;
    virtual AsciiChar const* getPluginNamespace() const noexcept = 0;
};

class IPluginV3OneBuild : public IPluginCapability {
public:
    virtual int32_t configurePlugin(DynamicPluginTensorDesc const* in, int32_t nbInputs,
                                    DynamicPluginTensorDesc const* out, int32_t nbOutputs) noexcept = 0;
    virtual int32_t getOutputDataTypes(DataType* outputTypes, int32_t nbOutputs, DataType const* inputTypes,
                                       int32_t nbInputs) const noexcept = 0;
    virtual int32_t getOutputShapes(DimsExprs const* inputs, int32_t nbInputs, DimsExprs const* shapeInputs,
                                    int32_t nbShapeInputs, DimsExprs* outputs, int32_t nbOutputs,
                                    IExprBuilder& exprBuilder) noexcept = 0;
    virtual bool supportsFormatCombination(int32_t pos, DynamicPluginTensorDesc const* inOut, int32_t nbInputs,
                                           int32_t nbOutputs) noexcept = 0;
    virtual int32_t getNbOutputs() const noexcept = 0;
    virtual size_t getWorkspaceSize(DynamicPluginTensorDesc const* /*inputs*/, int32_t /*nbInputs*/,
                                    DynamicPluginTensorDesc const* /*outputs*/,
                                    int32_t /*nbOutputs*/) const noexcept
    {
        return 0;
    }
};

class IPluginV3OneRuntime : public IPluginCapability {
public:
    virtual int32_t onShapeChange(PluginTensorDesc const* in, int32_t nbInputs, PluginTensorDesc const* out,
                                  int32_t nbOutputs) noexcept = 0;
    virtual int32_t enqueue(PluginTensorDesc const* inputDesc, PluginTensorDesc const* outputDesc,
                            void const* const* inputs, void* const* outputs, void* workspace,
                            cudaStream_t stream) noexcept = 0;
    virtual IPluginV3* attachToContext(IPluginResourceContext* context) noexcept = 0;
    virtual PluginFieldCollection const* getFieldsToSerialize() noexcept = 0;
};

class IPluginCreatorInterface {
public:
    virtual ~IPluginCreatorInterface() = default;
};

class IPluginCreatorV3One : public IPluginCreatorInterface {
public:
    virtual IPluginV3* createPlugin(AsciiChar const* name, PluginFieldCollection const* fc,
                                    TensorRTPhase phase) noexcept = 0;
    virtual PluginFieldCollection const* getFieldNames() noexcept = 0;
    virtual AsciiChar const* getPluginName() const noexcept = 0;
    virtual AsciiChar const* getPluginVersion() const noexcept = 0;
    virtual AsciiChar const* getPluginNamespace() const noexcept = 0;
};

}  // namespace nvinfer1

// Static registration: one registrar object per creator type.
#define REGISTER_TENSORRT_PLUGIN(name) static name ww_stub_registrar_##name
