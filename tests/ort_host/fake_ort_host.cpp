// fake_ort_host.cpp -- TEST INFRASTRUCTURE: a minimal stand-in for the parts of
// ONNX Runtime that a compiling plugin EP talks to, so the tests can drive
// libdoe_ort_ep.so through its real C ABI without an ORT runtime (none exists
// on the build or GPU machines).
//
// It implements, on in-memory objects, the OrtApi / OrtEpApi members the EP
// calls: graph / node / value-info inspection with consumers and initializers,
// node attributes, EpGraphSupportInfo_AddNodesToFuse, the kernel context of a
// Compute call (inputs are caller-provided device pointers, the output is a
// caller-provided buffer), memory infos / devices, hardware devices and
// EpDevice creation, and sync-stream lookup.  Every other OrtApi slot stays
// null: a call to one would crash the test, which is what a test should do.
//
// The test drives it through the flat fh_* functions at the end (ctypes).
#include <cstdint>
#include <cstring>
#include <dlfcn.h>
#include <execinfo.h>
#include <signal.h>
#include <unistd.h>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "onnxruntime_c_api.h"

struct OrtStatus {
  OrtErrorCode code;
  std::string msg;
};
struct OrtTensorTypeAndShapeInfo {
  ONNXTensorElementDataType type = ONNX_TENSOR_ELEMENT_DATA_TYPE_UNDEFINED;
  std::vector<int64_t> dims;
};
struct OrtTypeInfo {
  OrtTensorTypeAndShapeInfo tensor;
};
struct OrtOpAttr {
  OrtOpAttrType type = ORT_OP_ATTR_UNDEFINED;
  int64_t i = 0;
  float f = 0.0f;
};
struct OrtMemoryDevice {
  OrtMemoryInfoDeviceType type = OrtMemoryInfoDeviceType_CPU;
  OrtDeviceMemoryType mem = OrtDeviceMemoryType_DEFAULT;
  uint32_t vendor = 0;
  uint32_t id = 0;
};
struct OrtMemoryInfo {
  std::string name;
  OrtMemoryDevice dev;
};
struct OrtValue {
  void* data = nullptr;
  ONNXTensorElementDataType type = ONNX_TENSOR_ELEMENT_DATA_TYPE_UNDEFINED;
  std::vector<int64_t> dims;
  OrtMemoryDevice dev;
};
struct OrtNode;
struct OrtValueInfo {
  std::string name;
  bool typed = false;
  OrtTypeInfo ti;
  std::vector<std::pair<const OrtNode*, int64_t>> consumers;
  bool graph_output = false;
  bool initializer = false;
  std::vector<uint8_t> init_data;
  OrtValue init_value;
};
struct OrtNode {
  std::string name, op, domain;
  std::vector<OrtValueInfo*> ins, outs;
  std::map<std::string, OrtOpAttr> attrs;
};
struct OrtGraph {
  std::vector<std::unique_ptr<OrtValueInfo>> value_store;
  std::vector<std::unique_ptr<OrtNode>> node_store;
  std::vector<const OrtNode*> nodes;
  std::vector<const OrtValueInfo*> inputs;
};
struct OrtEpGraphSupportInfo {
  std::vector<std::vector<const OrtNode*>> groups;
};
struct OrtHardwareDevice {
  OrtHardwareDeviceType type;
  uint32_t vendor;
  uint32_t device;
};
struct OrtEpDevice {
  const OrtHardwareDevice* hw = nullptr;
  std::vector<const OrtMemoryInfo*> allocator_infos;
};
struct OrtKeyValuePairs {
  std::vector<std::pair<std::string, std::string>> kv;
};
struct OrtNodeComputeContext {
  std::string name;
};
struct OrtSyncStream {
  OrtSyncStreamImpl* impl = nullptr;
};
struct OrtKernelContext {
  std::vector<OrtValue*> inputs;
  OrtValue output;
  size_t output_capacity = 0;
  bool output_taken = false;
  void* stream = nullptr;
};

namespace {

std::string g_last_error;

OrtStatus* make(OrtErrorCode c, const std::string& m) { return new OrtStatus{c, m}; }

size_t elem_size(ONNXTensorElementDataType t) {
  switch (t) {
    case ONNX_TENSOR_ELEMENT_DATA_TYPE_FLOAT: return 4;
    case ONNX_TENSOR_ELEMENT_DATA_TYPE_FLOAT16:
    case ONNX_TENSOR_ELEMENT_DATA_TYPE_BFLOAT16: return 2;
    case ONNX_TENSOR_ELEMENT_DATA_TYPE_INT32: return 4;
    case ONNX_TENSOR_ELEMENT_DATA_TYPE_INT64: return 8;
    case ONNX_TENSOR_ELEMENT_DATA_TYPE_INT8:
    case ONNX_TENSOR_ELEMENT_DATA_TYPE_UINT8: return 1;
    default: return 0;
  }
}

size_t count_of(const std::vector<int64_t>& d) {
  size_t n = 1;
  for (int64_t x : d) n *= (size_t)(x < 0 ? 0 : x);
  return n;
}

// ---- OrtApi members ---------------------------------------------------------
OrtErrorCode ORT_API_CALL GetErrorCode(const OrtStatus* s) noexcept { return s->code; }
const char* ORT_API_CALL GetErrorMessage(const OrtStatus* s) noexcept { return s->msg.c_str(); }
void ORT_API_CALL ReleaseStatus(OrtStatus* s) noexcept { delete s; }
OrtStatus* ORT_API_CALL CreateStatus(OrtErrorCode c, const char* m) noexcept { return make(c, m ? m : ""); }

OrtStatus* ORT_API_CALL GetValueInfoName(const OrtValueInfo* v, const char** out) noexcept {
  *out = v->name.c_str();
  return nullptr;
}
OrtStatus* ORT_API_CALL GetValueInfoTypeInfo(const OrtValueInfo* v, const OrtTypeInfo** out) noexcept {
  *out = v->typed ? &v->ti : nullptr;
  return nullptr;
}
OrtStatus* ORT_API_CALL GetOnnxTypeFromTypeInfo(const OrtTypeInfo*, ONNXType* out) noexcept {
  *out = ONNX_TYPE_TENSOR;
  return nullptr;
}
OrtStatus* ORT_API_CALL CastTypeInfoToTensorInfo(const OrtTypeInfo* t, const OrtTensorTypeAndShapeInfo** out) noexcept {
  *out = &t->tensor;
  return nullptr;
}
OrtStatus* ORT_API_CALL GetTensorElementType(const OrtTensorTypeAndShapeInfo* t, ONNXTensorElementDataType* out) noexcept {
  *out = t->type;
  return nullptr;
}
OrtStatus* ORT_API_CALL GetDimensionsCount(const OrtTensorTypeAndShapeInfo* t, size_t* out) noexcept {
  *out = t->dims.size();
  return nullptr;
}
OrtStatus* ORT_API_CALL GetDimensions(const OrtTensorTypeAndShapeInfo* t, int64_t* out, size_t n) noexcept {
  for (size_t i = 0; i < n && i < t->dims.size(); ++i) out[i] = t->dims[i];
  return nullptr;
}
OrtStatus* ORT_API_CALL GetTensorShapeElementCount(const OrtTensorTypeAndShapeInfo* t, size_t* out) noexcept {
  *out = count_of(t->dims);
  return nullptr;
}
OrtStatus* ORT_API_CALL Node_GetNumInputs(const OrtNode* n, size_t* out) noexcept {
  *out = n->ins.size();
  return nullptr;
}
OrtStatus* ORT_API_CALL Node_GetNumOutputs(const OrtNode* n, size_t* out) noexcept {
  *out = n->outs.size();
  return nullptr;
}
OrtStatus* ORT_API_CALL Node_GetInputs(const OrtNode* n, const OrtValueInfo** out, size_t k) noexcept {
  if (k < n->ins.size()) return make(ORT_INVALID_ARGUMENT, "Node_GetInputs: array too small");
  for (size_t i = 0; i < n->ins.size(); ++i) out[i] = n->ins[i];
  return nullptr;
}
OrtStatus* ORT_API_CALL Node_GetOutputs(const OrtNode* n, const OrtValueInfo** out, size_t k) noexcept {
  if (k < n->outs.size()) return make(ORT_INVALID_ARGUMENT, "Node_GetOutputs: array too small");
  for (size_t i = 0; i < n->outs.size(); ++i) out[i] = n->outs[i];
  return nullptr;
}
OrtStatus* ORT_API_CALL Node_GetName(const OrtNode* n, const char** out) noexcept {
  *out = n->name.c_str();
  return nullptr;
}
OrtStatus* ORT_API_CALL Node_GetOperatorType(const OrtNode* n, const char** out) noexcept {
  *out = n->op.c_str();
  return nullptr;
}
OrtStatus* ORT_API_CALL Node_GetDomain(const OrtNode* n, const char** out) noexcept {
  *out = n->domain.c_str();
  return nullptr;
}
OrtStatus* ORT_API_CALL Node_GetAttributeByName(const OrtNode* n, const char* name, const OrtOpAttr** out) noexcept {
  auto it = n->attrs.find(name);
  *out = it == n->attrs.end() ? nullptr : &it->second;
  return nullptr;
}
OrtStatus* ORT_API_CALL OpAttr_GetType(const OrtOpAttr* a, OrtOpAttrType* out) noexcept {
  *out = a->type;
  return nullptr;
}
OrtStatus* ORT_API_CALL ReadOpAttr(const OrtOpAttr* a, OrtOpAttrType t, void* data, size_t len, size_t* out) noexcept {
  if (t != a->type) return make(ORT_INVALID_ARGUMENT, "ReadOpAttr: type mismatch");
  if (t == ORT_OP_ATTR_INT && len >= 8) std::memcpy(data, &a->i, 8), *out = 8;
  else if (t == ORT_OP_ATTR_FLOAT && len >= 4) std::memcpy(data, &a->f, 4), *out = 4;
  else return make(ORT_INVALID_ARGUMENT, "ReadOpAttr: buffer too small");
  return nullptr;
}
OrtStatus* ORT_API_CALL Graph_GetNumNodes(const OrtGraph* g, size_t* out) noexcept {
  *out = g->nodes.size();
  return nullptr;
}
OrtStatus* ORT_API_CALL Graph_GetNodes(const OrtGraph* g, const OrtNode** out, size_t k) noexcept {
  if (k < g->nodes.size()) return make(ORT_INVALID_ARGUMENT, "Graph_GetNodes: array too small");
  for (size_t i = 0; i < g->nodes.size(); ++i) out[i] = g->nodes[i];
  return nullptr;
}
OrtStatus* ORT_API_CALL Graph_GetNumInputs(const OrtGraph* g, size_t* out) noexcept {
  *out = g->inputs.size();
  return nullptr;
}
OrtStatus* ORT_API_CALL Graph_GetInputs(const OrtGraph* g, const OrtValueInfo** out, size_t k) noexcept {
  if (k < g->inputs.size()) return make(ORT_INVALID_ARGUMENT, "Graph_GetInputs: array too small");
  for (size_t i = 0; i < g->inputs.size(); ++i) out[i] = g->inputs[i];
  return nullptr;
}
OrtStatus* ORT_API_CALL ValueInfo_IsConstantInitializer(const OrtValueInfo* v, bool* out) noexcept {
  *out = v->initializer;
  return nullptr;
}
OrtStatus* ORT_API_CALL ValueInfo_IsGraphOutput(const OrtValueInfo* v, bool* out) noexcept {
  *out = v->graph_output;
  return nullptr;
}
OrtStatus* ORT_API_CALL ValueInfo_GetValueNumConsumers(const OrtValueInfo* v, size_t* out) noexcept {
  *out = v->consumers.size();
  return nullptr;
}
OrtStatus* ORT_API_CALL ValueInfo_GetValueConsumers(const OrtValueInfo* v, const OrtNode** nodes, int64_t* idx,
                                                    size_t k) noexcept {
  if (k < v->consumers.size()) return make(ORT_INVALID_ARGUMENT, "ValueInfo_GetValueConsumers: array too small");
  for (size_t i = 0; i < v->consumers.size(); ++i) nodes[i] = v->consumers[i].first, idx[i] = v->consumers[i].second;
  return nullptr;
}
OrtStatus* ORT_API_CALL ValueInfo_GetInitializerValue(const OrtValueInfo* v, const OrtValue** out) noexcept {
  *out = v->initializer ? &v->init_value : nullptr;
  return nullptr;
}
OrtStatus* ORT_API_CALL KernelContext_GetInputCount(const OrtKernelContext* c, size_t* out) noexcept {
  *out = c->inputs.size();
  return nullptr;
}
OrtStatus* ORT_API_CALL KernelContext_GetOutputCount(const OrtKernelContext*, size_t* out) noexcept {
  *out = 1;
  return nullptr;
}
OrtStatus* ORT_API_CALL KernelContext_GetInput(const OrtKernelContext* c, size_t i, const OrtValue** out) noexcept {
  if (i >= c->inputs.size()) return make(ORT_INVALID_ARGUMENT, "KernelContext_GetInput: index out of range");
  *out = c->inputs[i];
  return nullptr;
}
OrtStatus* ORT_API_CALL KernelContext_GetOutput(OrtKernelContext* c, size_t i, const int64_t* dims, size_t n,
                                                OrtValue** out) noexcept {
  if (i != 0) return make(ORT_INVALID_ARGUMENT, "KernelContext_GetOutput: one output");
  c->output.dims.assign(dims, dims + n);
  if (count_of(c->output.dims) * elem_size(c->output.type) > c->output_capacity)
    return make(ORT_FAIL, "KernelContext_GetOutput: the output buffer is too small");
  c->output_taken = true;
  *out = &c->output;
  return nullptr;
}
OrtStatus* ORT_API_CALL KernelContext_GetGPUComputeStream(const OrtKernelContext* c, void** out) noexcept {
  *out = c->stream;
  return nullptr;
}
OrtStatus* ORT_API_CALL GetTensorTypeAndShape(const OrtValue* v, OrtTensorTypeAndShapeInfo** out) noexcept {
  *out = new OrtTensorTypeAndShapeInfo{v->type, v->dims};
  return nullptr;
}
void ORT_API_CALL ReleaseTensorTypeAndShapeInfo(OrtTensorTypeAndShapeInfo* t) noexcept { delete t; }
OrtStatus* ORT_API_CALL GetTensorData(const OrtValue* v, const void** out) noexcept {
  *out = v->data;
  return nullptr;
}
OrtStatus* ORT_API_CALL GetTensorMutableData(OrtValue* v, void** out) noexcept {
  *out = v->data;
  return nullptr;
}
OrtStatus* ORT_API_CALL GetTensorSizeInBytes(const OrtValue* v, size_t* out) noexcept {
  *out = count_of(v->dims) * elem_size(v->type);
  return nullptr;
}
void ORT_API_CALL CreateKeyValuePairs(OrtKeyValuePairs** out) { *out = new OrtKeyValuePairs(); }
OrtHardwareDeviceType ORT_API_CALL HardwareDevice_Type(const OrtHardwareDevice* d) noexcept { return d->type; }
uint32_t ORT_API_CALL HardwareDevice_VendorId(const OrtHardwareDevice* d) noexcept { return d->vendor; }
OrtStatus* ORT_API_CALL CreateMemoryInfo_V2(const char* name, OrtMemoryInfoDeviceType type, uint32_t vendor,
                                            int32_t id, OrtDeviceMemoryType mem, size_t, OrtAllocatorType,
                                            OrtMemoryInfo** out) noexcept {
  auto* m = new OrtMemoryInfo();
  m->name = name ? name : "";
  m->dev.type = type;
  m->dev.vendor = vendor;
  m->dev.id = (uint32_t)id;
  m->dev.mem = mem;
  *out = m;
  return nullptr;
}
void ORT_API_CALL ReleaseMemoryInfo(OrtMemoryInfo* m) noexcept { delete m; }

// ---- OrtEpApi members -------------------------------------------------------
OrtStatus* ORT_API_CALL CreateEpDevice(OrtEpFactory*, const OrtHardwareDevice* hw, const OrtKeyValuePairs*,
                                       const OrtKeyValuePairs*, OrtEpDevice** out) noexcept {
  auto* d = new OrtEpDevice();
  d->hw = hw;
  *out = d;
  return nullptr;
}
OrtStatus* ORT_API_CALL AddNodesToFuse(OrtEpGraphSupportInfo* s, const OrtNode* const* nodes, size_t n,
                                       const OrtNodeFusionOptions*) noexcept {
  s->groups.emplace_back(nodes, nodes + n);
  return nullptr;
}
const char* ORT_API_CALL NodeComputeContext_NodeName(const OrtNodeComputeContext* c) noexcept { return c->name.c_str(); }
OrtStatus* ORT_API_CALL EpDevice_AddAllocatorInfo(OrtEpDevice* d, const OrtMemoryInfo* m) noexcept {
  d->allocator_infos.push_back(m);
  return nullptr;
}
const OrtMemoryDevice* ORT_API_CALL MemoryInfo_GetMemoryDevice(const OrtMemoryInfo* m) noexcept { return &m->dev; }
const OrtMemoryDevice* ORT_API_CALL Value_GetMemoryDevice(const OrtValue* v) noexcept { return &v->dev; }
OrtMemoryInfoDeviceType ORT_API_CALL MemoryDevice_GetDeviceType(const OrtMemoryDevice* d) noexcept { return d->type; }
OrtDeviceMemoryType ORT_API_CALL MemoryDevice_GetMemoryType(const OrtMemoryDevice* d) noexcept { return d->mem; }
uint32_t ORT_API_CALL MemoryDevice_GetVendorId(const OrtMemoryDevice* d) noexcept { return d->vendor; }
uint32_t ORT_API_CALL MemoryDevice_GetDeviceId(const OrtMemoryDevice* d) noexcept { return d->id; }
const OrtSyncStreamImpl* ORT_API_CALL SyncStream_GetImpl(const OrtSyncStream* s) noexcept { return s->impl; }

OrtApi g_api;
OrtEpApi g_ep_api;
OrtApiBase g_base;

const OrtEpApi* ORT_API_CALL GetEpApi() noexcept { return &g_ep_api; }
const OrtApi* ORT_API_CALL GetApi(uint32_t version) noexcept { return version <= ORT_API_VERSION ? &g_api : nullptr; }
const char* ORT_API_CALL GetVersionString() noexcept { return "fake-ort-host"; }

void init_api() {
  static bool done = false;
  if (done) return;
  done = true;
  std::memset(&g_api, 0, sizeof(g_api));
  std::memset(&g_ep_api, 0, sizeof(g_ep_api));
  g_api.GetErrorCode = &GetErrorCode;
  g_api.GetErrorMessage = &GetErrorMessage;
  g_api.ReleaseStatus = &ReleaseStatus;
  g_api.CreateStatus = &CreateStatus;
  g_api.GetEpApi = &GetEpApi;
  g_api.GetValueInfoName = &GetValueInfoName;
  g_api.GetValueInfoTypeInfo = &GetValueInfoTypeInfo;
  g_api.GetOnnxTypeFromTypeInfo = &GetOnnxTypeFromTypeInfo;
  g_api.CastTypeInfoToTensorInfo = &CastTypeInfoToTensorInfo;
  g_api.GetTensorElementType = &GetTensorElementType;
  g_api.GetDimensionsCount = &GetDimensionsCount;
  g_api.GetDimensions = &GetDimensions;
  g_api.GetTensorShapeElementCount = &GetTensorShapeElementCount;
  g_api.Node_GetNumInputs = &Node_GetNumInputs;
  g_api.Node_GetNumOutputs = &Node_GetNumOutputs;
  g_api.Node_GetInputs = &Node_GetInputs;
  g_api.Node_GetOutputs = &Node_GetOutputs;
  g_api.Node_GetName = &Node_GetName;
  g_api.Node_GetOperatorType = &Node_GetOperatorType;
  g_api.Node_GetDomain = &Node_GetDomain;
  g_api.Node_GetAttributeByName = &Node_GetAttributeByName;
  g_api.OpAttr_GetType = &OpAttr_GetType;
  g_api.ReadOpAttr = &ReadOpAttr;
  g_api.Graph_GetNumNodes = &Graph_GetNumNodes;
  g_api.Graph_GetNodes = &Graph_GetNodes;
  g_api.Graph_GetNumInputs = &Graph_GetNumInputs;
  g_api.Graph_GetInputs = &Graph_GetInputs;
  g_api.ValueInfo_IsConstantInitializer = &ValueInfo_IsConstantInitializer;
  g_api.ValueInfo_IsGraphOutput = &ValueInfo_IsGraphOutput;
  g_api.ValueInfo_GetValueNumConsumers = &ValueInfo_GetValueNumConsumers;
  g_api.ValueInfo_GetValueConsumers = &ValueInfo_GetValueConsumers;
  g_api.ValueInfo_GetInitializerValue = &ValueInfo_GetInitializerValue;
  g_api.KernelContext_GetInputCount = &KernelContext_GetInputCount;
  g_api.KernelContext_GetOutputCount = &KernelContext_GetOutputCount;
  g_api.KernelContext_GetInput = &KernelContext_GetInput;
  g_api.KernelContext_GetOutput = &KernelContext_GetOutput;
  g_api.KernelContext_GetGPUComputeStream = &KernelContext_GetGPUComputeStream;
  g_api.GetTensorTypeAndShape = &GetTensorTypeAndShape;
  g_api.ReleaseTensorTypeAndShapeInfo = &ReleaseTensorTypeAndShapeInfo;
  g_api.GetTensorData = &GetTensorData;
  g_api.GetTensorMutableData = &GetTensorMutableData;
  g_api.GetTensorSizeInBytes = &GetTensorSizeInBytes;
  g_api.CreateKeyValuePairs = &CreateKeyValuePairs;
  g_api.HardwareDevice_Type = &HardwareDevice_Type;
  g_api.HardwareDevice_VendorId = &HardwareDevice_VendorId;
  g_api.CreateMemoryInfo_V2 = &CreateMemoryInfo_V2;
  g_api.ReleaseMemoryInfo = &ReleaseMemoryInfo;
  g_ep_api.CreateEpDevice = &CreateEpDevice;
  g_ep_api.EpGraphSupportInfo_AddNodesToFuse = &AddNodesToFuse;
  g_ep_api.NodeComputeContext_NodeName = &NodeComputeContext_NodeName;
  g_ep_api.EpDevice_AddAllocatorInfo = &EpDevice_AddAllocatorInfo;
  g_ep_api.MemoryInfo_GetMemoryDevice = &MemoryInfo_GetMemoryDevice;
  g_ep_api.Value_GetMemoryDevice = &Value_GetMemoryDevice;
  g_ep_api.MemoryDevice_GetDeviceType = &MemoryDevice_GetDeviceType;
  g_ep_api.MemoryDevice_GetMemoryType = &MemoryDevice_GetMemoryType;
  g_ep_api.MemoryDevice_GetVendorId = &MemoryDevice_GetVendorId;
  g_ep_api.MemoryDevice_GetDeviceId = &MemoryDevice_GetDeviceId;
  g_ep_api.SyncStream_GetImpl = &SyncStream_GetImpl;
  g_base.GetApi = &GetApi;
  g_base.GetVersionString = &GetVersionString;
}

// Turns an EP status into the host's last error (and a code to return).
int take(OrtStatus* s) {
  if (s == nullptr) return 0;
  g_last_error = s->msg;
  const int code = (int)s->code;
  delete s;
  return code == 0 ? -1 : code;
}

struct Compiled {
  std::unique_ptr<OrtGraph> sub;  // shares the parent's nodes and values
  OrtNodeComputeInfo* info = nullptr;
  void* state = nullptr;
  OrtNodeComputeContext ctx;
};

struct Host {
  void* dl = nullptr;
  OrtEpFactory* factory = nullptr;
  OrtEp* ep = nullptr;
  OrtHardwareDevice gpu{OrtHardwareDeviceType_GPU, 0x10DE, 0x2901};
  OrtHardwareDevice cpu{OrtHardwareDeviceType_CPU, 0, 0};
  OrtEpGraphSupportInfo support;
  std::vector<Compiled> compiled;
  OrtStatus* (*release_factory)(OrtEpFactory*) = nullptr;
};

}  // namespace

namespace {
// Prints the native frames of a crash (library + offset, for addr2line) to
// stderr, then lets the signal take its default course.
void on_fatal_signal(int sig) {
  void* frames[64];
  const int n = backtrace(frames, 64);
  const char msg[] = "fake_ort_host: fatal signal; native frames:\n";
  if (write(2, msg, sizeof(msg) - 1) < 0) {
  }
  backtrace_symbols_fd(frames, n, 2);
  signal(sig, SIG_DFL);
  raise(sig);
}
}  // namespace

extern "C" {

const char* fh_last_error() { return g_last_error.c_str(); }

void fh_install_crash_handler() {
  signal(SIGSEGV, on_fatal_signal);
  signal(SIGBUS, on_fatal_signal);
  signal(SIGABRT, on_fatal_signal);
}

// ---- graphs ------------------------------------------------------------------
OrtGraph* fh_graph_new() { return new OrtGraph(); }
void fh_graph_free(OrtGraph* g) { delete g; }

// A value: elem_type 0 (or rank < 0) leaves it untyped; kind 0 intermediate,
// 1 graph input, 2 graph output, 3 constant initializer.
int fh_value(OrtGraph* g, const char* name, int elem_type, int rank, const int64_t* dims, int kind) {
  auto v = std::make_unique<OrtValueInfo>();
  v->name = name;
  v->typed = elem_type != 0 && rank >= 0;
  v->ti.tensor.type = (ONNXTensorElementDataType)elem_type;
  if (rank > 0) v->ti.tensor.dims.assign(dims, dims + rank);
  v->graph_output = kind == 2;
  v->initializer = kind == 3;
  if (kind == 1) g->inputs.push_back(v.get());
  g->value_store.push_back(std::move(v));
  return (int)g->value_store.size() - 1;
}

int fh_set_initializer(OrtGraph* g, int value, const void* data, size_t bytes) {
  OrtValueInfo* v = g->value_store.at(value).get();
  v->init_data.assign((const uint8_t*)data, (const uint8_t*)data + bytes);
  v->init_value.data = v->init_data.data();
  v->init_value.type = v->ti.tensor.type;
  v->init_value.dims = v->ti.tensor.dims;
  return 0;
}

int fh_node(OrtGraph* g, const char* name, const char* op, const char* domain, int n_in, const int* ins, int n_out,
            const int* outs) {
  auto n = std::make_unique<OrtNode>();
  n->name = name;
  n->op = op;
  n->domain = domain ? domain : "";
  for (int i = 0; i < n_in; ++i) {
    OrtValueInfo* v = g->value_store.at(ins[i]).get();
    n->ins.push_back(v);
    v->consumers.emplace_back(n.get(), i);
  }
  for (int i = 0; i < n_out; ++i) n->outs.push_back(g->value_store.at(outs[i]).get());
  g->nodes.push_back(n.get());
  g->node_store.push_back(std::move(n));
  return (int)g->node_store.size() - 1;
}

int fh_attr_int(OrtGraph* g, int node, const char* name, int64_t v) {
  OrtOpAttr a;
  a.type = ORT_OP_ATTR_INT;
  a.i = v;
  g->node_store.at(node)->attrs[name] = a;
  return 0;
}
int fh_attr_float(OrtGraph* g, int node, const char* name, float v) {
  OrtOpAttr a;
  a.type = ORT_OP_ATTR_FLOAT;
  a.f = v;
  g->node_store.at(node)->attrs[name] = a;
  return 0;
}

// ---- the EP ------------------------------------------------------------------
// Loads the EP library and makes its factory and one EP for CUDA ordinal 0.
Host* fh_load(const char* path, const char* registered_name) {
  init_api();
  auto h = std::make_unique<Host>();
  h->dl = dlopen(path, RTLD_NOW | RTLD_LOCAL);
  if (!h->dl) {
    g_last_error = dlerror();
    return nullptr;
  }
  using Create = OrtStatus* (*)(const char*, const OrtApiBase*, const OrtLogger*, OrtEpFactory**, size_t, size_t*);
  auto create = (Create)dlsym(h->dl, "CreateEpFactories");
  h->release_factory = (OrtStatus * (*)(OrtEpFactory*)) dlsym(h->dl, "ReleaseEpFactory");
  if (!create || !h->release_factory) {
    g_last_error = "CreateEpFactories / ReleaseEpFactory not exported";
    return nullptr;
  }
  size_t n = 0;
  if (take(create(registered_name, &g_base, nullptr, &h->factory, 1, &n)) || n != 1) return nullptr;
  const OrtHardwareDevice* devs[] = {&h->gpu};
  if (take(h->factory->CreateEp(h->factory, devs, nullptr, 1, nullptr, nullptr, &h->ep))) return nullptr;
  return h.release();
}

void fh_unload(Host* h) {
  if (!h) return;
  for (Compiled& c : h->compiled) {
    if (c.state) c.info->ReleaseState(c.info, c.state);
    if (c.info) h->ep->ReleaseNodeComputeInfos(h->ep, &c.info, 1);
  }
  if (h->ep) h->factory->ReleaseEp(h->factory, h->ep);
  if (h->factory) h->release_factory(h->factory);
  delete h;  // the library stays loaded: its CUDA state outlives this host
}

const char* fh_ep_name(Host* h) { return h->ep->GetName(h->ep); }
const char* fh_factory_name(Host* h) { return h->factory->GetName(h->factory); }

// GetSupportedDevices over [cpu, gpu, gpu]: returns the EP devices made and
// the allocator infos the first one registered (vendor, device id).
int fh_supported_devices(Host* h, int* n_out, uint32_t* vendor, uint32_t* device_id, int* mem_type) {
  const OrtHardwareDevice* devs[] = {&h->cpu, &h->gpu, &h->gpu};
  OrtEpDevice* eps[4] = {};
  size_t n = 0;
  int rc = take(h->factory->GetSupportedDevices(h->factory, devs, 3, eps, 4, &n));
  *n_out = (int)n;
  if (n > 0 && !eps[0]->allocator_infos.empty()) {
    *vendor = eps[0]->allocator_infos[0]->dev.vendor;
    *device_id = eps[0]->allocator_infos[0]->dev.id;
    *mem_type = (int)eps[0]->allocator_infos[0]->dev.type;
  }
  for (size_t i = 0; i < n; ++i) delete eps[i];
  return rc;
}

// GetCapability: the number of fused groups claimed (or -1 on an error).
int fh_get_capability(Host* h, OrtGraph* g) {
  h->support.groups.clear();
  if (take(h->ep->GetCapability(h->ep, g, &h->support))) return -1;
  return (int)h->support.groups.size();
}

// Node indices (in `g`) of claimed group `i`; returns its size.
int fh_group(Host* h, OrtGraph* g, int i, int* nodes, int max) {
  const auto& grp = h->support.groups.at(i);
  int k = 0;
  for (const OrtNode* n : grp) {
    for (size_t j = 0; j < g->node_store.size(); ++j)
      if (g->node_store[j].get() == n && k < max) nodes[k++] = (int)j;
  }
  return (int)grp.size();
}

// Compile claimed group `i` as ORT would: a subgraph of its nodes whose
// inputs are the values they read that no member writes and that are not
// constant initializers.  Returns a compiled-node handle (>= 0) or -1.
int fh_compile(Host* h, OrtGraph* g, int i, const char* fused_name) {
  Compiled c;
  c.sub = std::make_unique<OrtGraph>();
  const auto& grp = h->support.groups.at(i);
  for (const OrtNode* n : grp) c.sub->nodes.push_back(n);
  for (const OrtNode* n : grp)
    for (OrtValueInfo* v : n->ins) {
      bool produced = false;
      for (const OrtNode* m : grp)
        for (OrtValueInfo* o : m->outs) produced |= o == v;
      bool seen = false;
      for (const OrtValueInfo* x : c.sub->inputs) seen |= x == v;
      if (!produced && !seen && !v->initializer) c.sub->inputs.push_back(v);
    }
  (void)g;
  OrtNode fused;
  fused.name = fused_name ? fused_name : "";
  const OrtGraph* graphs[] = {c.sub.get()};
  const OrtNode* fused_nodes[] = {&fused};
  OrtNodeComputeInfo* info = nullptr;
  OrtNode* ctx_node = nullptr;
  if (take(h->ep->Compile(h->ep, graphs, fused_nodes, 1, &info, &ctx_node))) return -1;
  c.info = info;
  c.ctx.name = fused.name;
  if (take(info->CreateState(info, &c.ctx, &c.state))) {
    h->ep->ReleaseNodeComputeInfos(h->ep, &c.info, 1);
    return -1;
  }
  h->compiled.push_back(std::move(c));
  return (int)h->compiled.size() - 1;
}

// Compute of compiled node `ci` with `n` device inputs (types, ranks and
// concatenated dims) into a device output buffer of `out_capacity` bytes and
// `out_type`; writes the output's rank and dims.  `stream`: the kernel
// context's GPU compute stream (null: the EP's own).
int fh_compute(Host* h, int ci, int n, void* const* data, const int* types, const int* ranks, const int64_t* dims,
               void* out, int out_type, size_t out_capacity, int* out_rank, int64_t* out_dims, void* stream) {
  Compiled& c = h->compiled.at(ci);
  OrtKernelContext k;
  std::vector<OrtValue> vals((size_t)n);
  const int64_t* d = dims;
  for (int i = 0; i < n; ++i) {
    vals[i].data = data[i];
    vals[i].type = (ONNXTensorElementDataType)types[i];
    vals[i].dims.assign(d, d + ranks[i]);
    d += ranks[i];
    k.inputs.push_back(&vals[i]);
  }
  k.output.data = out;
  k.output.type = (ONNXTensorElementDataType)out_type;
  k.output_capacity = out_capacity;
  k.stream = stream;
  int rc = take(c.info->Compute(c.info, c.state, &k));
  *out_rank = (int)k.output.dims.size();
  for (size_t i = 0; i < k.output.dims.size(); ++i) out_dims[i] = k.output.dims[i];
  return rc;
}

// ---- allocator, data transfer, sync stream ------------------------------------
// One round trip host -> device -> device -> host through the EP's allocator
// and data transfer, on the EP's sync stream and a notification; returns 0
// when the bytes come back equal.
int fh_device_roundtrip(Host* h, const void* src, void* dst, size_t bytes) {
  OrtMemoryInfo* mi = nullptr;
  CreateMemoryInfo_V2("DoeCuda", OrtMemoryInfoDeviceType_GPU, 0x10DE, 0, OrtDeviceMemoryType_DEFAULT, 256,
                      OrtDeviceAllocator, &mi);
  OrtAllocator* a = nullptr;
  if (take(h->factory->CreateAllocator(h->factory, mi, nullptr, &a)) || !a) return -1;
  void* d1 = a->Alloc(a, bytes);
  void* d2 = a->Alloc(a, bytes);
  if (!d1 || !d2) {
    g_last_error = "allocator returned null";
    return -1;
  }
  OrtDataTransferImpl* t = nullptr;
  if (take(h->factory->CreateDataTransfer(h->factory, &t)) || !t) return -1;
  OrtSyncStreamImpl* s = nullptr;
  if (!h->factory->IsStreamAware(h->factory)) {
    g_last_error = "factory is not stream aware";
    return -1;
  }
  if (take(h->factory->CreateSyncStreamForDevice(h->factory, &mi->dev, nullptr, &s)) || !s || !s->GetHandle(s)) {
    g_last_error = "no sync stream";
    return -1;
  }
  OrtSyncStream os{s};
  OrtMemoryDevice host{OrtMemoryInfoDeviceType_CPU, OrtDeviceMemoryType_DEFAULT, 0, 0};
  if (!t->CanCopy(t, &host, &mi->dev) || !t->CanCopy(t, &mi->dev, &host) || !t->CanCopy(t, &mi->dev, &mi->dev) ||
      t->CanCopy(t, &host, &host)) {
    g_last_error = "CanCopy answered wrong";
    return -1;
  }
  const std::vector<int64_t> shape{(int64_t)bytes};
  OrtValue vs{const_cast<void*>(src), ONNX_TENSOR_ELEMENT_DATA_TYPE_UINT8, shape, host};
  OrtValue v1{d1, ONNX_TENSOR_ELEMENT_DATA_TYPE_UINT8, shape, mi->dev};
  OrtValue v2{d2, ONNX_TENSOR_ELEMENT_DATA_TYPE_UINT8, shape, mi->dev};
  OrtValue vd{dst, ONNX_TENSOR_ELEMENT_DATA_TYPE_UINT8, shape, host};
  const OrtValue* srcs[] = {&vs, &v1, &v2};
  OrtValue* dsts[] = {&v1, &v2, &vd};
  OrtSyncStream* streams[] = {&os, &os, &os};
  int rc = 0;
  for (int i = 0; i < 3 && rc == 0; ++i) rc = take(t->CopyTensors(t, &srcs[i], &dsts[i], streams, 1));
  OrtSyncNotificationImpl* note = nullptr;
  if (rc == 0) rc = take(s->CreateNotification(s, &note));
  if (rc == 0) rc = take(note->Activate(note));
  if (rc == 0) rc = take(note->WaitOnHost(note));
  if (note) note->Release(note);
  s->Release(s);
  t->Release(t);
  a->Free(a, d1);
  a->Free(a, d2);
  h->factory->ReleaseAllocator(h->factory, a);
  ReleaseMemoryInfo(mi);
  if (rc == 0 && std::memcmp(src, dst, bytes) != 0) {
    g_last_error = "round trip changed the bytes";
    rc = -1;
  }
  return rc;
}

}  // extern "C"
