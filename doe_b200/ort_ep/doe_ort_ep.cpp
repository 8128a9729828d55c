// doe_ort_ep.cpp -- ONNX Runtime plugin execution provider over libdoe_cuda.so.
//
// Replaces the reference's host-loop plugin EP
// (runtime/bridge/onnxruntime-ep/src/doe_ort_ep_exports.cc, doe_ort_ep_factory.cc,
// doe_ort_ep.cc) with one whose claimed nodes run as sm_100a kernels on device
// tensors.  What is kept from the reference, for drop-in compatibility:
//   * the exports CreateEpFactories / ReleaseEpFactory
//     (doe_ort_ep_exports.cc:13-50) and the debug-counter exports with the same
//     struct layout (doe_ort_ep.h:10-59, doe_ort_ep_exports.cc:52-61);
//   * the runtime API floor 23 (doe_ort_ep_api_version.h:9);
//   * the node kinds it claims and their static-shape rules
//     (GetSupportedNodeSpec, doe_ort_ep.cc:762-1002), the fusions
//     MatMul->Add(->Relu), Add->Relu and Gemm->Relu->Gemm with single-consumer
//     chains (doe_ort_ep.cc:1004-1395, 2615-2717), the per-kind input order of
//     a compiled group (doe_ort_ep.cc:1202-1395), and the runtime shape checks
//     and their messages (doe_ort_ep.cc:1847-1897).
// What changes: the factory hands ORT a CUDA device allocator, a data
// transfer (host <-> device, device <-> device) and a CUDA sync stream, where
// the reference returns none (doe_ort_ep_factory.cc:177-223), so ORT keeps
// claimed subgraphs' tensors in HBM; Compute launches libdoe_cuda kernels on
// the stream ORT gives the kernel context.  Two node types of a bf16 Llama
// decoder graph are claimed as well: SimplifiedLayerNormalization with f32 X
// and bf16 scale (doe_rmsnorm_bf16) and a bf16 MatMul by a constant
// initializer (doe_linear_bf16, the weight transposed once at Compile).
//
// Errors: every ORT entry point catches the internal Fail exception and
// returns an OrtStatus made by the ORT API; no exception crosses the ABI.
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdint>
#include <cstring>
#include <memory>
#include <mutex>
#include <new>
#include <sstream>
#include <string>
#include <string_view>
#include <unordered_map>
#include <unordered_set>
#include <vector>

#include "doe_cuda.h"
#include "onnxruntime_c_api.h"  // includes onnxruntime_ep_c_api.h

#define DOE_EP_EXPORT extern "C" __attribute__((visibility("default")))

namespace doeep {

constexpr uint32_t kApiFloor = 23;  // doe_ort_ep_api_version.h:9
constexpr uint32_t kNvidiaVendorId = 0x10DE;
constexpr const char* kDefaultName = "DoeExecutionProvider";
constexpr const char* kVendor = "Doe";
constexpr const char* kVersion = "0.1.0-cuda-sm100a";
constexpr const char* kCompatibility = "doe-ort-cuda-sm100a-ep-v1";
constexpr const char* kMemoryName = "DoeCuda";
constexpr float kLayerNormEpsilon = 1e-5f;  // doe_ort_ep.cc:52

// ---------------------------------------------------------------------------
// Debug counters: the reference's struct, field for field (doe_ort_ep.h:10-59),
// so its session smoke test reads them unchanged.
struct DebugCounters {
  uint64_t get_capability_calls, claimed_nodes, claimed_identity_nodes, claimed_add_nodes,
      claimed_relu_nodes, claimed_sigmoid_nodes, claimed_tanh_nodes, claimed_gelu_nodes,
      claimed_matmul_nodes, claimed_gemm_nodes, claimed_softmax_nodes, claimed_layernorm_nodes,
      claimed_concat_nodes, compile_calls, compiled_identity_groups, compiled_add_groups,
      compiled_relu_groups, compiled_sigmoid_groups, compiled_tanh_groups, compiled_gelu_groups,
      compiled_matmul_groups, compiled_gemm_groups, compiled_gemm_relu_gemm_groups,
      compiled_matmul_add_groups, compiled_matmul_add_relu_groups, compiled_add_relu_groups,
      compiled_softmax_groups, compiled_layernorm_groups, compiled_concat_groups, create_state_calls,
      compute_calls, compute_identity_calls, compute_add_calls, compute_relu_calls,
      compute_sigmoid_calls, compute_tanh_calls, compute_gelu_calls, compute_matmul_calls,
      compute_gemm_calls, compute_gemm_relu_gemm_calls, compute_matmul_add_calls,
      compute_matmul_add_relu_calls, compute_add_relu_calls, compute_softmax_calls,
      compute_layernorm_calls, compute_concat_calls, release_state_calls;
};
constexpr size_t kNumCounters = sizeof(DebugCounters) / sizeof(uint64_t);
std::atomic<uint64_t> g_counters[kNumCounters];
// The decoder-block kinds have no field in the reference struct: counted here.
std::atomic<uint64_t> g_decoder_claimed{0}, g_decoder_computed{0};

#define DOE_COUNTER(field) g_counters[offsetof(DebugCounters, field) / sizeof(uint64_t)]
void bump(std::atomic<uint64_t>& c, uint64_t n = 1) { c.fetch_add(n, std::memory_order_relaxed); }

// ---------------------------------------------------------------------------
enum class Kind {
  kIdentity, kAdd, kRelu, kSigmoid, kTanh, kGelu, kMatMul, kGemm, kGemmReluGemm, kMatMulAdd,
  kMatMulAddRelu, kAddRelu, kSoftmax, kLayerNorm, kConcat,
  kRmsNormBf16,  // SimplifiedLayerNormalization, X f32, scale / Y bf16
  kLinearBf16    // MatMul bf16 x constant bf16 weight
};

const char* kind_name(Kind k) {  // CompiledOpKindName (doe_ort_ep.cc:183-217)
  switch (k) {
    case Kind::kIdentity: return "Identity";
    case Kind::kAdd: return "Add";
    case Kind::kRelu: return "Relu";
    case Kind::kSigmoid: return "Sigmoid";
    case Kind::kTanh: return "Tanh";
    case Kind::kGelu: return "Gelu";
    case Kind::kMatMul: return "MatMul";
    case Kind::kGemm: return "Gemm";
    case Kind::kGemmReluGemm: return "Gemm->Relu->Gemm";
    case Kind::kMatMulAdd: return "MatMul->Add";
    case Kind::kMatMulAddRelu: return "MatMul->Add->Relu";
    case Kind::kAddRelu: return "Add->Relu";
    case Kind::kSoftmax: return "Softmax";
    case Kind::kLayerNorm: return "LayerNormalization";
    case Kind::kConcat: return "Concat";
    case Kind::kRmsNormBf16: return "SimplifiedLayerNormalization";
    case Kind::kLinearBf16: return "MatMul(bf16)";
  }
  return "unknown";
}

// Node counts, claim / compile / compute counters of a kind.
struct KindCounters {
  size_t nodes;
  std::atomic<uint64_t>* claimed;
  std::atomic<uint64_t>* compiled;
  std::atomic<uint64_t>* computed;
};
KindCounters counters_of(Kind k) {
  switch (k) {
    case Kind::kIdentity: return {1, &DOE_COUNTER(claimed_identity_nodes), &DOE_COUNTER(compiled_identity_groups), &DOE_COUNTER(compute_identity_calls)};
    case Kind::kAdd: return {1, &DOE_COUNTER(claimed_add_nodes), &DOE_COUNTER(compiled_add_groups), &DOE_COUNTER(compute_add_calls)};
    case Kind::kRelu: return {1, &DOE_COUNTER(claimed_relu_nodes), &DOE_COUNTER(compiled_relu_groups), &DOE_COUNTER(compute_relu_calls)};
    case Kind::kSigmoid: return {1, &DOE_COUNTER(claimed_sigmoid_nodes), &DOE_COUNTER(compiled_sigmoid_groups), &DOE_COUNTER(compute_sigmoid_calls)};
    case Kind::kTanh: return {1, &DOE_COUNTER(claimed_tanh_nodes), &DOE_COUNTER(compiled_tanh_groups), &DOE_COUNTER(compute_tanh_calls)};
    case Kind::kGelu: return {1, &DOE_COUNTER(claimed_gelu_nodes), &DOE_COUNTER(compiled_gelu_groups), &DOE_COUNTER(compute_gelu_calls)};
    case Kind::kMatMul: return {1, &DOE_COUNTER(claimed_matmul_nodes), &DOE_COUNTER(compiled_matmul_groups), &DOE_COUNTER(compute_matmul_calls)};
    case Kind::kGemm: return {1, &DOE_COUNTER(claimed_gemm_nodes), &DOE_COUNTER(compiled_gemm_groups), &DOE_COUNTER(compute_gemm_calls)};
    // fused groups: their member nodes are counted per operator type in
    // claim_group (IncrementClaimCounters, doe_ort_ep.cc:277-331)
    case Kind::kGemmReluGemm: return {3, nullptr, &DOE_COUNTER(compiled_gemm_relu_gemm_groups), &DOE_COUNTER(compute_gemm_relu_gemm_calls)};
    case Kind::kMatMulAdd: return {2, nullptr, &DOE_COUNTER(compiled_matmul_add_groups), &DOE_COUNTER(compute_matmul_add_calls)};
    case Kind::kMatMulAddRelu: return {3, nullptr, &DOE_COUNTER(compiled_matmul_add_relu_groups), &DOE_COUNTER(compute_matmul_add_relu_calls)};
    case Kind::kAddRelu: return {2, nullptr, &DOE_COUNTER(compiled_add_relu_groups), &DOE_COUNTER(compute_add_relu_calls)};
    case Kind::kSoftmax: return {1, &DOE_COUNTER(claimed_softmax_nodes), &DOE_COUNTER(compiled_softmax_groups), &DOE_COUNTER(compute_softmax_calls)};
    case Kind::kLayerNorm: return {1, &DOE_COUNTER(claimed_layernorm_nodes), &DOE_COUNTER(compiled_layernorm_groups), &DOE_COUNTER(compute_layernorm_calls)};
    case Kind::kConcat: return {1, &DOE_COUNTER(claimed_concat_nodes), &DOE_COUNTER(compiled_concat_groups), &DOE_COUNTER(compute_concat_calls)};
    case Kind::kRmsNormBf16:
    case Kind::kLinearBf16: return {1, &g_decoder_claimed, nullptr, &g_decoder_computed};
  }
  return {0, nullptr, nullptr, nullptr};
}

// Claim counters of a group: the nodes in all, and each member node under its
// operator type (a Gemm->Relu->Gemm group is two Gemm nodes and one Relu).
void claim_group(Kind k) {
  const KindCounters kc = counters_of(k);
  bump(DOE_COUNTER(claimed_nodes), kc.nodes);
  switch (k) {
    case Kind::kGemmReluGemm:
      bump(DOE_COUNTER(claimed_gemm_nodes), 2);
      bump(DOE_COUNTER(claimed_relu_nodes));
      break;
    case Kind::kMatMulAddRelu:
      bump(DOE_COUNTER(claimed_relu_nodes));
      [[fallthrough]];
    case Kind::kMatMulAdd:
      bump(DOE_COUNTER(claimed_matmul_nodes));
      bump(DOE_COUNTER(claimed_add_nodes));
      break;
    case Kind::kAddRelu:
      bump(DOE_COUNTER(claimed_add_nodes));
      bump(DOE_COUNTER(claimed_relu_nodes));
      break;
    default:
      bump(*kc.claimed);
  }
}

// ---------------------------------------------------------------------------
// Error plumbing.
struct Fail {
  OrtErrorCode code;
  std::string msg;
};
[[noreturn]] void fail(OrtErrorCode code, const std::string& msg) { throw Fail{code, msg}; }

struct Api {
  const OrtApiBase* base = nullptr;
  const OrtApi* ort = nullptr;
  const OrtEpApi* ep = nullptr;
  const OrtLogger* logger = nullptr;

  // Throws the status's code and message (releasing it) if it is an error.
  void ok(OrtStatus* st) const {
    if (st == nullptr) return;
    Fail f{ort->GetErrorCode(st), ort->GetErrorMessage(st)};
    ort->ReleaseStatus(st);
    throw f;
  }
};

template <class F>
OrtStatus* guarded(const Api& api, F&& body) noexcept {
  try {
    body();
    return nullptr;
  } catch (const Fail& f) {
    return api.ort ? api.ort->CreateStatus(f.code, ("Doe ORT plugin EP: " + f.msg).c_str()) : nullptr;
  } catch (const std::bad_alloc&) {
    return api.ort ? api.ort->CreateStatus(ORT_FAIL, "Doe ORT plugin EP: out of host memory") : nullptr;
  } catch (...) {
    return api.ort ? api.ort->CreateStatus(ORT_FAIL, "Doe ORT plugin EP: unexpected exception") : nullptr;
  }
}

void cuda_ok(cudaError_t e, const char* what) {
  if (e != cudaSuccess) fail(ORT_FAIL, std::string(what) + ": " + cudaGetErrorString(e));
}

void doe_ok(int rc, const char* what) {
  if (rc == DOE_OK) return;
  const char* msg = doe_cuda_op_last_error();
  fail(rc == DOE_INVALID_ARGUMENT ? ORT_INVALID_ARGUMENT : ORT_FAIL,
       std::string(what) + " failed (" + std::to_string(rc) + "): " + (msg ? msg : ""));
}

std::string shape_str(const std::vector<int64_t>& d) {  // ShapeString (doe_ort_ep.cc:433-444)
  std::ostringstream s;
  s << '[';
  for (size_t i = 0; i < d.size(); ++i) s << (i ? ", " : "") << d[i];
  s << ']';
  return s.str();
}

// ---------------------------------------------------------------------------
// Graph inspection.
struct Tensor {
  const OrtValueInfo* vi = nullptr;
  std::string name;
  ONNXTensorElementDataType type = ONNX_TENSOR_ELEMENT_DATA_TYPE_UNDEFINED;
  std::vector<int64_t> dims;
  bool known = false;  // a tensor with a static shape
};

Tensor describe(const Api& api, const OrtValueInfo* vi) {
  Tensor t;
  t.vi = vi;
  if (vi == nullptr) return t;
  const char* name = nullptr;
  api.ok(api.ort->GetValueInfoName(vi, &name));
  t.name = name ? name : "";
  const OrtTypeInfo* ti = nullptr;
  api.ok(api.ort->GetValueInfoTypeInfo(vi, &ti));
  if (ti == nullptr) return t;
  ONNXType ot = ONNX_TYPE_UNKNOWN;
  api.ok(api.ort->GetOnnxTypeFromTypeInfo(ti, &ot));
  if (ot != ONNX_TYPE_TENSOR) return t;
  const OrtTensorTypeAndShapeInfo* si = nullptr;
  api.ok(api.ort->CastTypeInfoToTensorInfo(ti, &si));
  if (si == nullptr) return t;
  api.ok(api.ort->GetTensorElementType(si, &t.type));
  size_t rank = 0;
  api.ok(api.ort->GetDimensionsCount(si, &rank));
  t.dims.assign(rank, 0);
  if (rank) api.ok(api.ort->GetDimensions(si, t.dims.data(), rank));
  t.known = std::all_of(t.dims.begin(), t.dims.end(), [](int64_t d) { return d >= 0; });
  return t;
}

std::vector<const OrtValueInfo*> node_values(const Api& api, const OrtNode* n, bool inputs) {
  size_t count = 0;
  api.ok(inputs ? api.ort->Node_GetNumInputs(n, &count) : api.ort->Node_GetNumOutputs(n, &count));
  std::vector<const OrtValueInfo*> v(count, nullptr);
  if (count) api.ok(inputs ? api.ort->Node_GetInputs(n, v.data(), count) : api.ort->Node_GetOutputs(n, v.data(), count));
  return v;
}

std::vector<const OrtNode*> graph_nodes(const Api& api, const OrtGraph* g) {
  size_t count = 0;
  api.ok(api.ort->Graph_GetNumNodes(g, &count));
  std::vector<const OrtNode*> v(count, nullptr);
  if (count) api.ok(api.ort->Graph_GetNodes(g, v.data(), count));
  return v;
}

std::vector<const OrtValueInfo*> graph_inputs(const Api& api, const OrtGraph* g) {
  size_t count = 0;
  api.ok(api.ort->Graph_GetNumInputs(g, &count));
  std::vector<const OrtValueInfo*> v(count, nullptr);
  if (count) api.ok(api.ort->Graph_GetInputs(g, v.data(), count));
  return v;
}

// The attribute `name` of a node, if present and of `type`; a present
// attribute of another type makes the node unsupported (nullopt-like false).
template <class T>
bool read_attr(const Api& api, const OrtNode* n, const char* name, OrtOpAttrType type, T* out, bool* wrong_type) {
  *wrong_type = false;
  const OrtOpAttr* a = nullptr;
  api.ok(api.ort->Node_GetAttributeByName(n, name, &a));
  if (a == nullptr) return false;
  OrtOpAttrType t = ORT_OP_ATTR_UNDEFINED;
  api.ok(api.ort->OpAttr_GetType(a, &t));
  if (t != type) {
    *wrong_type = true;
    return false;
  }
  size_t got = 0;
  api.ok(api.ort->ReadOpAttr(a, type, out, sizeof(T), &got));
  return got != 0;
}

bool onnx_domain(const char* d) {  // IsSupportedOnnxDomain (doe_ort_ep.cc:269-275)
  return d == nullptr || std::string_view(d).empty() || std::string_view(d) == "ai.onnx";
}

struct NodeSpec {
  const OrtNode* node = nullptr;
  Kind kind = Kind::kIdentity;
  std::string name;
  std::vector<Tensor> in, out;
  int64_t axis = 0;          // Concat axis (normalised), LayerNorm / RMSNorm axis
  float epsilon = kLayerNormEpsilon;
};

bool is_f32(const Tensor& t) { return t.known && t.type == ONNX_TENSOR_ELEMENT_DATA_TYPE_FLOAT; }
bool is_bf16(const Tensor& t) { return t.known && t.type == ONNX_TENSOR_ELEMENT_DATA_TYPE_BFLOAT16; }
bool same(const Tensor& a, const Tensor& b) { return a.type == b.type && a.dims == b.dims; }
bool rank2(const Tensor& t) { return t.dims.size() == 2; }

// The product shape [m, n] of [m, k] x [k, n] f32 matrices, if they are ones.
bool product_shape(const Tensor& a, const Tensor& b, Tensor* out) {
  if (!rank2(a) || !rank2(b) || a.type != b.type || a.dims[1] != b.dims[0]) return false;
  out->type = a.type;
  out->dims = {a.dims[0], b.dims[1]};
  out->known = true;
  return true;
}

// Whether an output that the graph left untyped or shapeless may take the
// inferred product shape (MatMul / Gemm outputs, doe_ort_ep.cc:917-951).
void settle_product_output(Tensor* out, const Tensor& inferred, bool* ok) {
  const bool usable = out->known && out->type == ONNX_TENSOR_ELEMENT_DATA_TYPE_FLOAT && rank2(*out);
  if (usable) {
    *ok = *ok && same(*out, inferred);
  } else {
    const OrtValueInfo* vi = out->vi;
    std::string name = out->name;
    *out = inferred;
    out->vi = vi;
    out->name = name;
  }
}

bool is_constant_initializer(const Api& api, const OrtValueInfo* vi) {
  bool c = false;
  api.ok(api.ort->ValueInfo_IsConstantInitializer(vi, &c));
  return c;
}

// GetSupportedNodeSpec (doe_ort_ep.cc:762-1002) plus the two decoder kinds.
bool classify(const Api& api, const OrtNode* node, NodeSpec* s) {
  *s = NodeSpec{};
  s->node = node;
  const char* name = nullptr;
  api.ok(api.ort->Node_GetName(node, &name));
  s->name = name ? name : "";
  const char* op = nullptr;
  api.ok(api.ort->Node_GetOperatorType(node, &op));
  const char* domain = nullptr;
  api.ok(api.ort->Node_GetDomain(node, &domain));
  if (op == nullptr) return false;
  const std::string_view o(op);
  const bool onnx = onnx_domain(domain);
  const bool ms = domain && std::string_view(domain) == "com.microsoft";
  size_t want = 0;
  if (onnx && o == "Identity") s->kind = Kind::kIdentity, want = 1;
  else if (onnx && o == "Add") s->kind = Kind::kAdd, want = 2;
  else if (onnx && o == "Relu") s->kind = Kind::kRelu, want = 1;
  else if (onnx && o == "Sigmoid") s->kind = Kind::kSigmoid, want = 1;
  else if (onnx && o == "Tanh") s->kind = Kind::kTanh, want = 1;
  else if (onnx && o == "Gelu") s->kind = Kind::kGelu, want = 1;
  else if (onnx && o == "MatMul") s->kind = Kind::kMatMul, want = 2;
  else if (onnx && o == "Gemm") s->kind = Kind::kGemm, want = 3;
  else if (onnx && o == "Softmax") s->kind = Kind::kSoftmax, want = 1;
  else if (onnx && o == "LayerNormalization") s->kind = Kind::kLayerNorm, want = 2;
  else if (onnx && o == "Concat") s->kind = Kind::kConcat, want = 2;
  else if ((onnx || ms) && o == "SimplifiedLayerNormalization") s->kind = Kind::kRmsNormBf16, want = 2;
  else return false;

  const auto ins = node_values(api, node, true);
  const auto outs = node_values(api, node, false);
  if (ins.size() != want || outs.size() != 1) return false;
  for (const OrtValueInfo* vi : ins) s->in.push_back(describe(api, vi));
  for (const OrtValueInfo* vi : outs) s->out.push_back(describe(api, vi));

  // bf16 MatMul by a constant weight: the decoder's projections
  if (s->kind == Kind::kMatMul && is_bf16(s->in[0]) && is_bf16(s->in[1])) {
    Tensor y;
    if (!product_shape(s->in[0], s->in[1], &y)) return false;
    const int64_t m = y.dims[0], k = s->in[0].dims[1], n = y.dims[1];
    if (m < 1 || m > 32 || k % 64 != 0 || n % 128 != 0 || n > (1 << 21) || k < 64) return false;
    if (!is_constant_initializer(api, s->in[1].vi)) return false;
    if (s->out[0].known && !same(s->out[0], y)) return false;
    s->kind = Kind::kLinearBf16;
    return true;
  }
  if (s->kind == Kind::kRmsNormBf16) {
    const Tensor &x = s->in[0], &g = s->in[1], &y = s->out[0];
    if (!is_f32(x) || x.dims.empty() || !is_bf16(g) || !is_bf16(y) || y.dims != x.dims) return false;
    if (g.dims.size() != 1 || g.dims[0] != x.dims.back() || x.dims.back() % 4 != 0) return false;
    bool wrong = false;
    int64_t axis = -1;
    read_attr(api, node, "axis", ORT_OP_ATTR_INT, &axis, &wrong);
    if (wrong || (axis != -1 && axis != (int64_t)x.dims.size() - 1)) return false;
    float eps = kLayerNormEpsilon;
    read_attr(api, node, "epsilon", ORT_OP_ATTR_FLOAT, &eps, &wrong);
    if (wrong) return false;
    s->epsilon = eps;
    return true;
  }

  for (const Tensor& t : s->in)
    if (!is_f32(t)) return false;
  const bool product = s->kind == Kind::kMatMul || s->kind == Kind::kGemm;
  if (!product && !is_f32(s->out[0])) return false;

  switch (s->kind) {
    case Kind::kIdentity:
    case Kind::kRelu:
    case Kind::kSigmoid:
    case Kind::kTanh:
    case Kind::kGelu:
    case Kind::kSoftmax:
      return same(s->in[0], s->out[0]);
    case Kind::kAdd:
      return same(s->in[0], s->in[1]) && same(s->in[0], s->out[0]);
    case Kind::kLayerNorm:
      return !s->in[0].dims.empty() && same(s->in[0], s->out[0]) && s->in[1].dims.size() == 1 &&
             s->in[1].dims[0] == s->in[0].dims.back();
    case Kind::kConcat: {
      const Tensor &a = s->in[0], &b = s->in[1], &y = s->out[0];
      if (a.dims.empty() || a.dims.size() != b.dims.size() || a.dims.size() != y.dims.size()) return false;
      bool wrong = false;
      int64_t axis = 0;
      read_attr(api, node, "axis", ORT_OP_ATTR_INT, &axis, &wrong);
      if (wrong) fail(ORT_INVALID_GRAPH, "Concat expected an int attribute 'axis'");
      const int64_t r = (int64_t)a.dims.size();
      if (axis < 0) axis += r;
      if (axis < 0 || axis >= r) return false;
      for (int64_t i = 0; i < r; ++i)
        if (i != axis && (a.dims[i] != b.dims[i] || a.dims[i] != y.dims[i])) return false;
      s->axis = axis;
      return y.dims[axis] == a.dims[axis] + b.dims[axis];
    }
    case Kind::kMatMul: {
      Tensor y;
      bool ok = product_shape(s->in[0], s->in[1], &y);
      if (ok) settle_product_output(&s->out[0], y, &ok);
      return ok;
    }
    case Kind::kGemm: {
      // alpha = beta = 1, no transposes (HasSupportedGemmAttributes, doe_ort_ep.cc:575-599)
      bool wrong = false;
      float alpha = 1.0f, beta = 1.0f;
      int64_t ta = 0, tb = 0;
      read_attr(api, node, "alpha", ORT_OP_ATTR_FLOAT, &alpha, &wrong);
      if (wrong) fail(ORT_INVALID_GRAPH, "Gemm expected float attribute 'alpha'");
      read_attr(api, node, "beta", ORT_OP_ATTR_FLOAT, &beta, &wrong);
      if (wrong) fail(ORT_INVALID_GRAPH, "Gemm expected float attribute 'beta'");
      read_attr(api, node, "transA", ORT_OP_ATTR_INT, &ta, &wrong);
      if (wrong) fail(ORT_INVALID_GRAPH, "Gemm expected int attribute 'transA'");
      read_attr(api, node, "transB", ORT_OP_ATTR_INT, &tb, &wrong);
      if (wrong) fail(ORT_INVALID_GRAPH, "Gemm expected int attribute 'transB'");
      if (alpha != 1.0f || beta != 1.0f || ta != 0 || tb != 0) return false;
      Tensor y;
      bool ok = product_shape(s->in[0], s->in[1], &y) && same(y, s->in[2]);
      if (ok) settle_product_output(&s->out[0], y, &ok);
      return ok;
    }
    default:
      return false;
  }
}

// The single consumer of a node's only output, with the input slot it reads,
// when that output is not a graph output and feeds exactly one node that is
// not claimed yet (the fusion precondition, doe_ort_ep.cc:1004-1061).
bool single_consumer(const Api& api, const NodeSpec& p, const std::unordered_set<const OrtNode*>& claimed,
                     const OrtNode** consumer, int64_t* slot) {
  if (p.out.size() != 1 || p.out[0].vi == nullptr) return false;
  bool graph_output = false;
  api.ok(api.ort->ValueInfo_IsGraphOutput(p.out[0].vi, &graph_output));
  if (graph_output) return false;
  size_t n = 0;
  api.ok(api.ort->ValueInfo_GetValueNumConsumers(p.out[0].vi, &n));
  if (n != 1) return false;
  const OrtNode* c = nullptr;
  int64_t idx = -1;
  api.ok(api.ort->ValueInfo_GetValueConsumers(p.out[0].vi, &c, &idx, 1));
  if (c == nullptr || claimed.count(c)) return false;
  *consumer = c;
  *slot = idx;
  return true;
}

// A fused group: its kind, nodes and the names of its inputs in the order
// Compute reads them (doe_ort_ep.cc:1202-1236, 1380-1395).
struct Group {
  Kind kind = Kind::kIdentity;
  std::vector<const OrtNode*> nodes;
  std::vector<std::string> inputs;
  std::string default_name;
  int64_t axis = 0;
  float epsilon = kLayerNormEpsilon;
  const OrtValueInfo* weight = nullptr;  // kLinearBf16: the constant weight
};

Group single(const NodeSpec& s) {
  Group g;
  g.kind = s.kind;
  g.nodes = {s.node};
  g.default_name = s.name.empty() ? kind_name(s.kind) : s.name;
  g.axis = s.axis;
  g.epsilon = s.epsilon;
  if (s.kind == Kind::kLinearBf16) {
    g.inputs = {s.in[0].name};
    g.weight = s.in[1].vi;
  } else {
    for (const Tensor& t : s.in) g.inputs.push_back(t.name);
  }
  return g;
}

// Extends a group rooted at `root` by the fusions the reference makes.
Group fuse(const Api& api, const NodeSpec& root, const std::unordered_set<const OrtNode*>& claimed) {
  Group g = single(root);
  const OrtNode* c = nullptr;
  int64_t slot = -1;
  NodeSpec next;
  auto relu_after = [&](const NodeSpec& p, NodeSpec* relu) {
    const OrtNode* rc = nullptr;
    int64_t rs = -1;
    return single_consumer(api, p, claimed, &rc, &rs) && rs == 0 && classify(api, rc, relu) &&
           relu->kind == Kind::kRelu;
  };
  if (root.kind == Kind::kMatMul) {
    // MatMul -> Add (either Add input) [-> Relu]
    if (!single_consumer(api, root, claimed, &c, &slot) || slot < 0 || slot > 1) return g;
    if (!classify(api, c, &next) || next.kind != Kind::kAdd) return g;
    const Tensor& mm = root.out[0];
    if (!same(next.in[0], mm) || !same(next.out[0], mm)) return g;
    g.kind = Kind::kMatMulAdd;
    g.default_name = "doe_matmul_add";
    g.nodes = {root.node, next.node};
    g.inputs = {root.in[0].name, root.in[1].name, next.in[slot == 0 ? 1 : 0].name};
    NodeSpec relu;
    if (relu_after(next, &relu)) {
      g.kind = Kind::kMatMulAddRelu;
      g.default_name = "doe_matmul_add_relu";
      g.nodes.push_back(relu.node);
    }
  } else if (root.kind == Kind::kAdd) {
    NodeSpec relu;
    if (relu_after(root, &relu)) {
      g.kind = Kind::kAddRelu;
      g.default_name = "doe_add_relu";
      g.nodes = {root.node, relu.node};
    }
  } else if (root.kind == Kind::kGemm) {
    // Gemm -> Relu -> Gemm (the relu output as the second Gemm's input 0)
    NodeSpec relu;
    if (!relu_after(root, &relu)) return g;
    if (!single_consumer(api, relu, claimed, &c, &slot) || slot != 0) return g;
    if (!classify(api, c, &next) || next.kind != Kind::kGemm) return g;
    g.kind = Kind::kGemmReluGemm;
    g.default_name = "doe_gemm_relu_gemm";
    g.nodes = {root.node, relu.node, next.node};
    g.inputs = {root.in[0].name, root.in[1].name, root.in[2].name, next.in[1].name, next.in[2].name};
  }
  return g;
}

// AnalyzeSupportedGraph (doe_ort_ep.cc:1451-1669): the group a fused subgraph
// handed to Compile forms -- the one GetCapability claimed from its first node.
bool analyze(const Api& api, const OrtGraph* graph, Group* out) {
  const auto nodes = graph_nodes(api, graph);
  if (nodes.empty() || nodes.size() > 3) return false;
  std::unordered_set<const OrtNode*> members(nodes.begin(), nodes.end());
  for (const OrtNode* n : nodes) {
    NodeSpec s;
    if (!classify(api, n, &s)) return false;
    // the group's root is the node whose chain covers the whole subgraph
    Group g = nodes.size() == 1 ? single(s) : fuse(api, s, {});
    if (g.nodes.size() != nodes.size()) continue;
    if (!std::all_of(g.nodes.begin(), g.nodes.end(), [&](const OrtNode* x) { return members.count(x); })) continue;
    *out = std::move(g);
    return true;
  }
  return false;
}

// ---------------------------------------------------------------------------
// Device memory, data transfer and streams.
struct Stream;

struct DeviceAllocator : OrtAllocator {
  const Api* api;
  OrtMemoryInfo* info;
  int device;
};

void* ORT_API_CALL alloc_impl(OrtAllocator* self, size_t size) noexcept {
  auto* a = static_cast<DeviceAllocator*>(self);
  void* p = nullptr;
  if (cudaSetDevice(a->device) != cudaSuccess || cudaMalloc(&p, size ? size : 1) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  return p;
}
void ORT_API_CALL free_impl(OrtAllocator* self, void* p) noexcept {
  auto* a = static_cast<DeviceAllocator*>(self);
  if (p) {
    cudaSetDevice(a->device);
    cudaFree(p);
  }
}
const OrtMemoryInfo* ORT_API_CALL info_impl(const OrtAllocator* self) noexcept {
  return static_cast<const DeviceAllocator*>(self)->info;
}
OrtStatus* ORT_API_CALL stats_impl(const OrtAllocator* self, OrtKeyValuePairs** out) noexcept {
  const Api& api = *static_cast<const DeviceAllocator*>(self)->api;
  return guarded(api, [&] {
    if (out) api.ort->CreateKeyValuePairs(out);
  });
}

constexpr uint64_t kStreamMagic = 0x646f652d73747265ull;  // "doe-stre"

struct Stream : OrtSyncStreamImpl {
  uint64_t magic = kStreamMagic;
  const Api* api = nullptr;
  cudaStream_t handle = nullptr;
  int device = 0;
};

struct Notification : OrtSyncNotificationImpl {
  const Api* api = nullptr;
  Stream* producer = nullptr;
  cudaEvent_t event = nullptr;
};

// The CUDA stream of an ORT sync stream this EP created (null otherwise).
cudaStream_t cuda_stream_of(const Api& api, OrtSyncStream* s) {
  if (s == nullptr || api.ep == nullptr) return nullptr;
  const OrtSyncStreamImpl* impl = api.ep->SyncStream_GetImpl(s);
  const Stream* st = static_cast<const Stream*>(impl);
  return st && st->magic == kStreamMagic ? st->handle : nullptr;
}

void ORT_API_CALL notification_release(OrtSyncNotificationImpl* self) noexcept {
  auto* n = static_cast<Notification*>(self);
  if (n->event) cudaEventDestroy(n->event);
  delete n;
}
OrtStatus* ORT_API_CALL notification_activate(OrtSyncNotificationImpl* self) noexcept {
  auto* n = static_cast<Notification*>(self);
  return guarded(*n->api, [&] { cuda_ok(cudaEventRecord(n->event, n->producer->handle), "cudaEventRecord"); });
}
OrtStatus* ORT_API_CALL notification_wait_device(OrtSyncNotificationImpl* self, OrtSyncStream* consumer) noexcept {
  auto* n = static_cast<Notification*>(self);
  return guarded(*n->api, [&] {
    cudaStream_t c = cuda_stream_of(*n->api, consumer);
    if (c) cuda_ok(cudaStreamWaitEvent(c, n->event, 0), "cudaStreamWaitEvent");
    else cuda_ok(cudaEventSynchronize(n->event), "cudaEventSynchronize");  // a stream of another EP
  });
}
OrtStatus* ORT_API_CALL notification_wait_host(OrtSyncNotificationImpl* self) noexcept {
  auto* n = static_cast<Notification*>(self);
  return guarded(*n->api, [&] { cuda_ok(cudaEventSynchronize(n->event), "cudaEventSynchronize"); });
}

void ORT_API_CALL stream_release(OrtSyncStreamImpl* self) noexcept {
  auto* s = static_cast<Stream*>(self);
  if (s->handle) {
    cudaSetDevice(s->device);
    cudaStreamSynchronize(s->handle);
    cudaStreamDestroy(s->handle);
  }
  delete s;
}
void* ORT_API_CALL stream_handle(OrtSyncStreamImpl* self) noexcept { return static_cast<Stream*>(self)->handle; }
OrtStatus* ORT_API_CALL stream_notification(OrtSyncStreamImpl* self, OrtSyncNotificationImpl** out) noexcept {
  auto* s = static_cast<Stream*>(self);
  return guarded(*s->api, [&] {
    auto n = std::make_unique<Notification>();
    std::memset(static_cast<OrtSyncNotificationImpl*>(n.get()), 0, sizeof(OrtSyncNotificationImpl));
    n->ort_version_supported = ORT_API_VERSION;
    n->Release = &notification_release;
    n->Activate = &notification_activate;
    n->WaitOnDevice = &notification_wait_device;
    n->WaitOnHost = &notification_wait_host;
    n->api = s->api;
    n->producer = s;
    cuda_ok(cudaSetDevice(s->device), "cudaSetDevice");
    cuda_ok(cudaEventCreateWithFlags(&n->event, cudaEventDisableTiming), "cudaEventCreate");
    *out = n.release();
  });
}
// Work queued on a CUDA stream is submitted already: nothing to flush.
OrtStatus* ORT_API_CALL stream_flush(OrtSyncStreamImpl*) noexcept { return nullptr; }
OrtStatus* ORT_API_CALL stream_run_end(OrtSyncStreamImpl*) noexcept { return nullptr; }

Stream* make_stream(const Api* api, int device) {
  auto s = std::make_unique<Stream>();
  std::memset(static_cast<OrtSyncStreamImpl*>(s.get()), 0, sizeof(OrtSyncStreamImpl));
  s->ort_version_supported = ORT_API_VERSION;
  s->Release = &stream_release;
  s->GetHandle = &stream_handle;
  s->CreateNotification = &stream_notification;
  s->Flush = &stream_flush;
  s->OnSessionRunEnd = &stream_run_end;
  s->api = api;
  s->device = device;
  cuda_ok(cudaSetDevice(device), "cudaSetDevice");
  cuda_ok(cudaStreamCreateWithFlags(&s->handle, cudaStreamNonBlocking), "cudaStreamCreate");
  return s.release();
}

struct Transfer : OrtDataTransferImpl {
  const Api* api;
};

bool our_device(const Api& api, const OrtMemoryDevice* d) {
  return api.ep->MemoryDevice_GetDeviceType(d) == OrtMemoryInfoDeviceType_GPU &&
         api.ep->MemoryDevice_GetVendorId(d) == kNvidiaVendorId;
}
bool host_device(const Api& api, const OrtMemoryDevice* d) {
  return api.ep->MemoryDevice_GetDeviceType(d) == OrtMemoryInfoDeviceType_CPU;
}

void ORT_API_CALL transfer_release(OrtDataTransferImpl* self) noexcept { delete static_cast<Transfer*>(self); }
bool ORT_API_CALL transfer_can_copy(const OrtDataTransferImpl* self, const OrtMemoryDevice* src,
                                    const OrtMemoryDevice* dst) noexcept {
  const Api& api = *static_cast<const Transfer*>(self)->api;
  const bool s_gpu = our_device(api, src), d_gpu = our_device(api, dst);
  return (s_gpu || d_gpu) && (s_gpu || host_device(api, src)) && (d_gpu || host_device(api, dst));
}
OrtStatus* ORT_API_CALL transfer_copy(OrtDataTransferImpl* self, const OrtValue** src, OrtValue** dst,
                                      OrtSyncStream** streams, size_t n) noexcept {
  const Api& api = *static_cast<Transfer*>(self)->api;
  return guarded(api, [&] {
    for (size_t i = 0; i < n; ++i) {
      size_t bytes = 0, dst_bytes = 0;
      api.ok(api.ort->GetTensorSizeInBytes(src[i], &bytes));
      api.ok(api.ort->GetTensorSizeInBytes(dst[i], &dst_bytes));
      if (bytes != dst_bytes) fail(ORT_INVALID_ARGUMENT, "CopyTensors: source and destination sizes differ");
      const void* s = nullptr;
      void* d = nullptr;
      api.ok(api.ort->GetTensorData(src[i], &s));
      api.ok(api.ort->GetTensorMutableData(dst[i], &d));
      if (bytes == 0) continue;
      const bool s_gpu = our_device(api, api.ep->Value_GetMemoryDevice(src[i]));
      const bool d_gpu = our_device(api, api.ep->Value_GetMemoryDevice(dst[i]));
      const cudaMemcpyKind kind = s_gpu && d_gpu ? cudaMemcpyDeviceToDevice
                                  : s_gpu       ? cudaMemcpyDeviceToHost
                                                : cudaMemcpyHostToDevice;
      cudaStream_t st = streams ? cuda_stream_of(api, streams[i]) : nullptr;
      if (st) cuda_ok(cudaMemcpyAsync(d, s, bytes, kind, st), "cudaMemcpyAsync");
      else cuda_ok(cudaMemcpy(d, s, bytes, kind), "cudaMemcpy");
    }
  });
}

// ---------------------------------------------------------------------------
// Compiled groups.
struct Ep;
cudaStream_t fallback_stream(Ep* ep);
struct ComputeState {
  std::string node_name;
  void* workspace = nullptr;  // per-state scratch (GemmReluGemm hidden activations)
  size_t workspace_bytes = 0;
  int device = 0;
  ~ComputeState() {
    if (workspace) {
      cudaSetDevice(device);
      cudaFree(workspace);
    }
  }
  void* scratch(size_t bytes) {
    if (bytes <= workspace_bytes) return workspace;
    if (workspace) cudaFree(workspace);
    workspace = nullptr;
    workspace_bytes = 0;
    cuda_ok(cudaMalloc(&workspace, bytes), "cudaMalloc(workspace)");
    workspace_bytes = bytes;
    return workspace;
  }
};

struct ComputeInfo : OrtNodeComputeInfo {
  const Api* api = nullptr;
  Group group;
  std::string node_name;
  std::vector<size_t> slots;  // kernel-context input index of each logical input
  int device = 0;
  struct Ep* ep = nullptr;  // owner: its stream serves Compute when ORT gives none
  // kLinearBf16: the weight transposed to [n, k] on the device, its sizes
  // and the zeroed linear workspace
  void* weight = nullptr;
  void* linear_ws = nullptr;
  int64_t n_out = 0, k_in = 0;
  ~ComputeInfo() {
    cudaSetDevice(device);
    if (weight) cudaFree(weight);
    if (linear_ws) cudaFree(linear_ws);
  }
};

struct In {
  const void* data = nullptr;
  std::vector<int64_t> dims;
  ONNXTensorElementDataType type = ONNX_TENSOR_ELEMENT_DATA_TYPE_UNDEFINED;
  size_t count = 0;
};

In kernel_input(const ComputeInfo& ci, OrtKernelContext* ctx, size_t logical) {
  const Api& api = *ci.api;
  if (logical >= ci.slots.size())
    fail(ORT_INVALID_GRAPH, std::string(kind_name(ci.group.kind)) + " slice has no input " + std::to_string(logical));
  const OrtValue* v = nullptr;
  api.ok(api.ort->KernelContext_GetInput(ctx, ci.slots[logical], &v));
  if (v == nullptr) fail(ORT_INVALID_GRAPH, "null input tensor at index " + std::to_string(ci.slots[logical]));
  In in;
  OrtTensorTypeAndShapeInfo* ti = nullptr;
  api.ok(api.ort->GetTensorTypeAndShape(v, &ti));
  std::unique_ptr<OrtTensorTypeAndShapeInfo, void (*)(OrtTensorTypeAndShapeInfo*)> hold(
      ti, api.ort->ReleaseTensorTypeAndShapeInfo);
  api.ok(api.ort->GetTensorElementType(ti, &in.type));
  size_t rank = 0;
  api.ok(api.ort->GetDimensionsCount(ti, &rank));
  in.dims.assign(rank, 0);
  if (rank) api.ok(api.ort->GetDimensions(ti, in.dims.data(), rank));
  for (int64_t d : in.dims)
    if (d < 0) fail(ORT_INVALID_GRAPH, "requires concrete runtime tensor shapes");
  api.ok(api.ort->GetTensorShapeElementCount(ti, &in.count));
  api.ok(api.ort->GetTensorData(v, &in.data));
  if (in.data == nullptr && in.count) fail(ORT_INVALID_GRAPH, "null tensor data for an input");
  return in;
}

void* kernel_output(const ComputeInfo& ci, OrtKernelContext* ctx, const std::vector<int64_t>& dims) {
  const Api& api = *ci.api;
  OrtValue* v = nullptr;
  api.ok(api.ort->KernelContext_GetOutput(ctx, 0, dims.empty() ? nullptr : dims.data(), dims.size(), &v));
  if (v == nullptr) fail(ORT_FAIL, "failed to allocate an output tensor");
  void* p = nullptr;
  api.ok(api.ort->GetTensorMutableData(v, &p));
  return p;
}

void need_f32(const ComputeInfo& ci, const In& t) {
  if (t.type != ONNX_TENSOR_ELEMENT_DATA_TYPE_FLOAT)
    fail(ORT_NOT_IMPLEMENTED, std::string(kind_name(ci.group.kind)) + " slice supports float32 tensors only");
}

// ValidateSameRuntimeShape (doe_ort_ep.cc:1847-1862).
void same_shape(const ComputeInfo& ci, const char* ln, const std::vector<int64_t>& l, const char* rn,
                const std::vector<int64_t>& r) {
  if (l == r) return;
  fail(ORT_INVALID_GRAPH, std::string(kind_name(ci.group.kind)) + " slice requires exact-shape float32 tensors; " +
                              ln + " has shape " + shape_str(l) + " while " + rn + " has shape " + shape_str(r) + ".");
}

// ValidateRuntimeMatMulShape (doe_ort_ep.cc:1864-1897): [m, n] of a x b.
std::vector<int64_t> matmul_shape(const In& a, const In& b) {
  if (a.dims.size() != 2 || b.dims.size() != 2)
    fail(ORT_INVALID_GRAPH, "MatMul slice requires rank-2 float32 inputs; input0 has shape " + shape_str(a.dims) +
                                " and input1 has shape " + shape_str(b.dims) + ".");
  if (a.dims[1] != b.dims[0])
    fail(ORT_INVALID_GRAPH, "MatMul slice requires exact matrix inner dimensions; input0 has shape " +
                                shape_str(a.dims) + " and input1 has shape " + shape_str(b.dims) + ".");
  return {a.dims[0], b.dims[1]};
}

doe_launch launch_on(cudaStream_t s, void* ws = nullptr, size_t ws_bytes = 0) {
  doe_launch l;
  l.stream = s;
  l.workspace = ws;
  l.workspace_bytes = ws_bytes;
  l.status = nullptr;
  return l;
}

void compute(ComputeInfo& ci, ComputeState* state, OrtKernelContext* ctx) {
  const Api& api = *ci.api;
  size_t n_in = 0, n_out = 0;
  api.ok(api.ort->KernelContext_GetInputCount(ctx, &n_in));
  api.ok(api.ort->KernelContext_GetOutputCount(ctx, &n_out));
  if (n_in < ci.slots.size())
    fail(ORT_INVALID_GRAPH, std::string(kind_name(ci.group.kind)) + " slice expects " +
                                std::to_string(ci.slots.size()) + " inputs but received " + std::to_string(n_in) + ".");
  if (n_out != 1)
    fail(ORT_INVALID_GRAPH, std::string(kind_name(ci.group.kind)) + " slice expects exactly 1 outputs but received " +
                                std::to_string(n_out) + ".");
  cuda_ok(cudaSetDevice(ci.device), "cudaSetDevice");
  void* sp = nullptr;
  OrtStatus* st = api.ort->KernelContext_GetGPUComputeStream(ctx, &sp);
  if (st != nullptr) {
    api.ort->ReleaseStatus(st);
    sp = nullptr;
  }
  cudaStream_t stream = sp ? static_cast<cudaStream_t>(sp) : fallback_stream(ci.ep);
  doe_launch l = launch_on(stream);
  const Kind k = ci.group.kind;
  switch (k) {
    case Kind::kIdentity:
    case Kind::kRelu:
    case Kind::kSigmoid:
    case Kind::kTanh:
    case Kind::kGelu: {
      In x = kernel_input(ci, ctx, 0);
      need_f32(ci, x);
      void* y = kernel_output(ci, ctx, x.dims);
      const uint32_t op = k == Kind::kIdentity ? DOE_EP_IDENTITY
                          : k == Kind::kRelu   ? DOE_EP_RELU
                          : k == Kind::kSigmoid ? DOE_EP_SIGMOID
                          : k == Kind::kTanh    ? DOE_EP_TANH
                                                : DOE_EP_GELU;
      doe_ok(doe_ep_unary_f32(op, (const float*)x.data, (float*)y, x.count, &l), "doe_ep_unary_f32");
      break;
    }
    case Kind::kAdd:
    case Kind::kAddRelu: {
      In a = kernel_input(ci, ctx, 0), b = kernel_input(ci, ctx, 1);
      need_f32(ci, a);
      need_f32(ci, b);
      same_shape(ci, "input0", a.dims, "input1", b.dims);
      void* y = kernel_output(ci, ctx, a.dims);
      doe_ok(doe_ep_binary_f32(k == Kind::kAdd ? DOE_EP_ADD : DOE_EP_ADD_RELU, (const float*)a.data,
                               (const float*)b.data, (float*)y, a.count, &l),
             "doe_ep_binary_f32");
      break;
    }
    case Kind::kMatMul:
    case Kind::kGemm:
    case Kind::kMatMulAdd:
    case Kind::kMatMulAddRelu: {
      In a = kernel_input(ci, ctx, 0), b = kernel_input(ci, ctx, 1);
      need_f32(ci, a);
      need_f32(ci, b);
      const auto yd = matmul_shape(a, b);
      const float* addend = nullptr;
      if (k != Kind::kMatMul) {
        In c = kernel_input(ci, ctx, 2);
        need_f32(ci, c);
        same_shape(ci, "matmul_output", yd, k == Kind::kGemm ? "gemm_bias" : "add_input", c.dims);
        addend = (const float*)c.data;
      }
      void* y = kernel_output(ci, ctx, yd);
      doe_ok(doe_ep_matmul_f32((const float*)a.data, (const float*)b.data, addend, (float*)y, (uint32_t)yd[0],
                               (uint32_t)a.dims[1], (uint32_t)yd[1],
                               k == Kind::kMatMulAddRelu ? DOE_EP_MATMUL_RELU : 0u, &l),
             "doe_ep_matmul_f32");
      break;
    }
    case Kind::kGemmReluGemm: {
      In x = kernel_input(ci, ctx, 0), w1 = kernel_input(ci, ctx, 1), b1 = kernel_input(ci, ctx, 2),
         w2 = kernel_input(ci, ctx, 3), b2 = kernel_input(ci, ctx, 4);
      for (const In* t : {&x, &w1, &b1, &w2, &b2}) need_f32(ci, *t);
      const auto hd = matmul_shape(x, w1);
      same_shape(ci, "hidden_gemm_output", hd, "hidden_bias", b1.dims);
      In h;
      h.dims = hd;
      const auto od = matmul_shape(h, w2);
      same_shape(ci, "output_gemm_output", od, "output_bias", b2.dims);
      const size_t ws = doe_ep_gemm_relu_gemm_workspace_bytes((uint32_t)hd[0], (uint32_t)hd[1]);
      l = launch_on(stream, state->scratch(ws), ws);
      void* y = kernel_output(ci, ctx, od);
      doe_ok(doe_ep_gemm_relu_gemm_f32((const float*)x.data, (const float*)w1.data, (const float*)b1.data,
                                       (const float*)w2.data, (const float*)b2.data, (float*)y, (uint32_t)hd[0],
                                       (uint32_t)x.dims[1], (uint32_t)hd[1], (uint32_t)od[1], &l),
             "doe_ep_gemm_relu_gemm_f32");
      break;
    }
    case Kind::kSoftmax: {
      In x = kernel_input(ci, ctx, 0);
      need_f32(ci, x);
      if (x.dims.empty()) fail(ORT_INVALID_GRAPH, "Softmax requires a tensor with rank >= 1.");
      void* y = kernel_output(ci, ctx, x.dims);
      const uint64_t cols = (uint64_t)x.dims.back();
      doe_ok(doe_ep_softmax_f32((const float*)x.data, (float*)y, cols ? x.count / cols : 0, (uint32_t)cols, &l),
             "doe_ep_softmax_f32");
      break;
    }
    case Kind::kLayerNorm: {
      In x = kernel_input(ci, ctx, 0), s = kernel_input(ci, ctx, 1);
      need_f32(ci, x);
      need_f32(ci, s);
      if (x.dims.empty()) fail(ORT_INVALID_GRAPH, "LayerNormalization requires a tensor with rank >= 1.");
      const uint64_t cols = (uint64_t)x.dims.back();
      if (s.count != cols) fail(ORT_INVALID_GRAPH, "LayerNormalization scale length must match the last input dimension.");
      void* y = kernel_output(ci, ctx, x.dims);
      doe_ok(doe_ep_layernorm_f32((const float*)x.data, (const float*)s.data, kLayerNormEpsilon, (float*)y,
                                  cols ? x.count / cols : 0, (uint32_t)cols, &l),
             "doe_ep_layernorm_f32");
      break;
    }
    case Kind::kConcat: {
      In a = kernel_input(ci, ctx, 0), b = kernel_input(ci, ctx, 1);
      need_f32(ci, a);
      need_f32(ci, b);
      const int64_t r = (int64_t)a.dims.size();
      const int64_t ax = ci.group.axis;
      if (r == 0 || (int64_t)b.dims.size() != r || ax >= r)
        fail(ORT_INVALID_GRAPH, "Concat requires two inputs of the same rank >= 1.");
      for (int64_t i = 0; i < r; ++i)
        if (i != ax && a.dims[i] != b.dims[i])
          fail(ORT_INVALID_GRAPH, "Concat inputs must match in every non-axis dimension.");
      std::vector<int64_t> yd = a.dims;
      yd[ax] += b.dims[ax];
      uint64_t outer = 1, inner = 1;
      for (int64_t i = 0; i < ax; ++i) outer *= (uint64_t)a.dims[i];
      for (int64_t i = ax + 1; i < r; ++i) inner *= (uint64_t)a.dims[i];
      void* y = kernel_output(ci, ctx, yd);
      doe_ok(doe_ep_concat_f32((const float*)a.data, (const float*)b.data, (float*)y, outer, (uint64_t)a.dims[ax],
                               (uint64_t)b.dims[ax], inner, &l),
             "doe_ep_concat_f32");
      break;
    }
    case Kind::kRmsNormBf16: {
      In x = kernel_input(ci, ctx, 0), g = kernel_input(ci, ctx, 1);
      if (x.type != ONNX_TENSOR_ELEMENT_DATA_TYPE_FLOAT || g.type != ONNX_TENSOR_ELEMENT_DATA_TYPE_BFLOAT16)
        fail(ORT_NOT_IMPLEMENTED, "SimplifiedLayerNormalization takes float32 X and bfloat16 scale");
      if (x.dims.empty() || g.count != (size_t)x.dims.back())
        fail(ORT_INVALID_GRAPH, "SimplifiedLayerNormalization scale length must match the last input dimension.");
      void* y = kernel_output(ci, ctx, x.dims);
      const uint32_t cols = (uint32_t)x.dims.back();
      doe_ok(doe_rmsnorm_bf16((const float*)x.data, g.data, ci.group.epsilon, y, (uint32_t)(x.count / cols), cols, &l),
             "doe_rmsnorm_bf16");
      break;
    }
    case Kind::kLinearBf16: {
      In x = kernel_input(ci, ctx, 0);
      if (x.type != ONNX_TENSOR_ELEMENT_DATA_TYPE_BFLOAT16 || x.dims.size() != 2 || x.dims[1] != ci.k_in ||
          x.dims[0] < 1 || x.dims[0] > 32)
        fail(ORT_INVALID_GRAPH, "MatMul(bf16) expects a [1..32, " + std::to_string(ci.k_in) +
                                    "] bfloat16 input; got " + shape_str(x.dims));
      void* y = kernel_output(ci, ctx, {x.dims[0], ci.n_out});
      doe_linear_out o;
      std::memset(&o, 0, sizeof(o));
      o.out[0] = y;
      o.width[0] = (uint32_t)ci.n_out;
      o.dtype = DOE_DTYPE_BF16;
      o.epilogue = DOE_LINEAR_STORE;
      const uint64_t wsb = doe_linear_workspace_bytes((uint32_t)ci.n_out, (uint32_t)ci.k_in);
      l = launch_on(stream, ci.linear_ws, wsb);
      doe_ok(doe_linear_bf16(x.data, ci.weight, (uint32_t)x.dims[0], (uint32_t)ci.n_out, (uint32_t)ci.k_in, &o, &l),
             "doe_linear_bf16");
      break;
    }
  }
}

OrtStatus* ORT_API_CALL create_state(OrtNodeComputeInfo* self, OrtNodeComputeContext* cc, void** out) noexcept {
  auto* ci = static_cast<ComputeInfo*>(self);
  return guarded(*ci->api, [&] {
    if (out == nullptr) fail(ORT_INVALID_ARGUMENT, "requires a compute_state output pointer");
    bump(DOE_COUNTER(create_state_calls));
    auto st = std::make_unique<ComputeState>();
    const char* nn = ci->api->ep && cc ? ci->api->ep->NodeComputeContext_NodeName(cc) : nullptr;
    st->node_name = nn ? nn : ci->node_name;
    st->device = ci->device;
    *out = st.release();
  });
}

OrtStatus* ORT_API_CALL compute_impl(OrtNodeComputeInfo* self, void* state, OrtKernelContext* ctx) noexcept {
  auto* ci = static_cast<ComputeInfo*>(self);
  return guarded(*ci->api, [&] {
    if (ctx == nullptr) fail(ORT_INVALID_ARGUMENT, "requires a kernel_context input");
    bump(DOE_COUNTER(compute_calls));
    bump(*counters_of(ci->group.kind).computed);
    compute(*ci, static_cast<ComputeState*>(state), ctx);
  });
}

void ORT_API_CALL release_state(OrtNodeComputeInfo*, void* state) noexcept {
  bump(DOE_COUNTER(release_state_calls));
  delete static_cast<ComputeState*>(state);
}

// A bf16 [k, n] initializer transposed to [n, k] in device memory.
void upload_weight(const Api& api, ComputeInfo* ci) {
  const OrtValue* w = nullptr;
  api.ok(api.ort->ValueInfo_GetInitializerValue(ci->group.weight, &w));
  if (w == nullptr) fail(ORT_INVALID_GRAPH, "MatMul(bf16) weight is not an initializer");
  OrtTensorTypeAndShapeInfo* ti = nullptr;
  api.ok(api.ort->GetTensorTypeAndShape(w, &ti));
  std::unique_ptr<OrtTensorTypeAndShapeInfo, void (*)(OrtTensorTypeAndShapeInfo*)> hold(
      ti, api.ort->ReleaseTensorTypeAndShapeInfo);
  int64_t dims[2] = {0, 0};
  size_t rank = 0;
  api.ok(api.ort->GetDimensionsCount(ti, &rank));
  if (rank != 2) fail(ORT_INVALID_GRAPH, "MatMul(bf16) weight must be rank 2");
  api.ok(api.ort->GetDimensions(ti, dims, 2));
  const void* data = nullptr;
  api.ok(api.ort->GetTensorData(w, &data));
  const int64_t k = dims[0], n = dims[1];
  std::vector<uint16_t> t((size_t)(k * n));
  const uint16_t* src = static_cast<const uint16_t*>(data);
  cudaPointerAttributes pa;
  std::vector<uint16_t> host;
  if (cudaPointerGetAttributes(&pa, data) == cudaSuccess && pa.type == cudaMemoryTypeDevice) {
    host.resize(t.size());  // an initializer ORT already placed on the device
    cuda_ok(cudaMemcpy(host.data(), data, t.size() * 2, cudaMemcpyDeviceToHost), "cudaMemcpy(weight)");
    src = host.data();
  }
  cudaGetLastError();
  for (int64_t r = 0; r < k; ++r)
    for (int64_t c = 0; c < n; ++c) t[(size_t)(c * k + r)] = src[(size_t)(r * n + c)];
  ci->n_out = n;
  ci->k_in = k;
  cuda_ok(cudaSetDevice(ci->device), "cudaSetDevice");
  cuda_ok(cudaMalloc(&ci->weight, t.size() * 2), "cudaMalloc(weight)");
  cuda_ok(cudaMemcpy(ci->weight, t.data(), t.size() * 2, cudaMemcpyHostToDevice), "cudaMemcpy(weight)");
  const uint64_t wsb = doe_linear_workspace_bytes((uint32_t)n, (uint32_t)k);
  cuda_ok(cudaMalloc(&ci->linear_ws, wsb), "cudaMalloc(linear workspace)");
  cuda_ok(cudaMemset(ci->linear_ws, 0, wsb), "cudaMemset(linear workspace)");
}

// ---------------------------------------------------------------------------
// The EP.
struct Ep : OrtEp {
  Api api;
  std::string name;
  int device = 0;
  std::mutex mu;
  cudaStream_t stream = nullptr;  // Compute's stream when ORT gives none (made at first use)
  ~Ep() {
    if (stream) {
      cudaSetDevice(device);
      cudaStreamDestroy(stream);
    }
  }
};

cudaStream_t fallback_stream(Ep* ep) {
  std::lock_guard<std::mutex> lock(ep->mu);
  if (ep->stream == nullptr) {
    cuda_ok(cudaSetDevice(ep->device), "cudaSetDevice");
    cuda_ok(cudaStreamCreateWithFlags(&ep->stream, cudaStreamNonBlocking), "cudaStreamCreate");
  }
  return ep->stream;
}

Ep& self_of(OrtEp* p) { return *static_cast<Ep*>(p); }

const char* ORT_API_CALL ep_name(const OrtEp* p) noexcept { return static_cast<const Ep*>(p)->name.c_str(); }

OrtStatus* ORT_API_CALL ep_get_capability(OrtEp* p, const OrtGraph* graph, OrtEpGraphSupportInfo* info) noexcept {
  Ep& ep = self_of(p);
  return guarded(ep.api, [&] {
    if (graph == nullptr || info == nullptr) fail(ORT_INVALID_ARGUMENT, "requires non-null graph and graph_support_info");
    if (ep.api.ep == nullptr) fail(ORT_NOT_IMPLEMENTED, "requires OrtEpApi to report graph support");
    bump(DOE_COUNTER(get_capability_calls));
    std::unordered_set<const OrtNode*> claimed;
    for (const OrtNode* n : graph_nodes(ep.api, graph)) {
      if (n == nullptr || claimed.count(n)) continue;
      NodeSpec s;
      if (!classify(ep.api, n, &s)) continue;
      Group g = fuse(ep.api, s, claimed);
      ep.api.ok(ep.api.ep->EpGraphSupportInfo_AddNodesToFuse(info, g.nodes.data(), g.nodes.size(), nullptr));
      claimed.insert(g.nodes.begin(), g.nodes.end());
      claim_group(g.kind);
    }
  });
}

void ORT_API_CALL ep_release_infos(OrtEp*, OrtNodeComputeInfo** infos, size_t n) noexcept {
  if (infos == nullptr) return;
  for (size_t i = 0; i < n; ++i) {
    delete static_cast<ComputeInfo*>(infos[i]);
    infos[i] = nullptr;
  }
}

OrtStatus* ORT_API_CALL ep_compile(OrtEp* p, const OrtGraph** graphs, const OrtNode** fused, size_t count,
                                   OrtNodeComputeInfo** infos, OrtNode** ctx_nodes) noexcept {
  Ep& ep = self_of(p);
  size_t done = 0;
  OrtStatus* st = guarded(ep.api, [&] {
    bump(DOE_COUNTER(compile_calls));
    if (count && (graphs == nullptr || infos == nullptr)) fail(ORT_INVALID_ARGUMENT, "requires graphs and node_compute_infos");
    for (size_t i = 0; i < count; ++i) {
      infos[i] = nullptr;
      if (ctx_nodes) ctx_nodes[i] = nullptr;
    }
    for (; done < count; ++done) {
      Group g;
      if (!analyze(ep.api, graphs[done], &g))
        fail(ORT_NOT_IMPLEMENTED, "asked to compile a graph outside the node kinds and fusions it claims");
      auto ci = std::make_unique<ComputeInfo>();
      std::memset(static_cast<OrtNodeComputeInfo*>(ci.get()), 0, sizeof(OrtNodeComputeInfo));
      ci->ort_version_supported = ORT_API_VERSION;
      ci->CreateState = &create_state;
      ci->Compute = &compute_impl;
      ci->ReleaseState = &release_state;
      ci->api = &ep.api;
      ci->device = ep.device;
      ci->ep = &ep;
      ci->group = g;
      // ResolveGraphInputBindings (doe_ort_ep.cc:1397-1449): logical inputs by name
      const auto gi = graph_inputs(ep.api, graphs[done]);
      std::vector<std::string> names;
      for (const OrtValueInfo* vi : gi) {
        const char* nm = nullptr;
        ep.api.ok(ep.api.ort->GetValueInfoName(vi, &nm));
        names.emplace_back(nm ? nm : "");
      }
      for (const std::string& want : g.inputs) {
        auto it = std::find(names.begin(), names.end(), want);
        if (it == names.end())
          fail(ORT_INVALID_GRAPH, std::string(kind_name(g.kind)) + " slice could not resolve fused graph input '" + want + "'.");
        ci->slots.push_back((size_t)(it - names.begin()));
      }
      if (g.kind == Kind::kLinearBf16) upload_weight(ep.api, ci.get());
      const OrtNode* name_src = fused && fused[done] ? fused[done] : g.nodes.front();
      const char* nn = nullptr;
      ep.api.ok(ep.api.ort->Node_GetName(name_src, &nn));
      ci->node_name = nn && nn[0] ? nn : g.default_name;
      if (KindCounters kc = counters_of(g.kind); kc.compiled) bump(*kc.compiled);
      infos[done] = ci.release();
    }
  });
  if (st != nullptr) ep_release_infos(p, infos, done);
  return st;
}

OrtStatus* ORT_API_CALL ep_layout(OrtEp* p, OrtEpDataLayout* layout) noexcept {
  Ep& ep = self_of(p);
  return guarded(ep.api, [&] {
    if (layout == nullptr) fail(ORT_INVALID_ARGUMENT, "requires a preferred_data_layout output");
    *layout = OrtEpDataLayout_NCHW;
  });
}
OrtStatus* ORT_API_CALL ep_run_start(OrtEp*, const OrtRunOptions*) noexcept { return nullptr; }
OrtStatus* ORT_API_CALL ep_run_end(OrtEp* p, const OrtRunOptions*, bool sync) noexcept {
  Ep& ep = self_of(p);
  return guarded(ep.api, [&] {
    std::lock_guard<std::mutex> lock(ep.mu);
    if (sync && ep.stream) {
      cuda_ok(cudaSetDevice(ep.device), "cudaSetDevice");
      cuda_ok(cudaStreamSynchronize(ep.stream), "cudaStreamSynchronize");
    }
  });
}
const char* ORT_API_CALL ep_compat(OrtEp*, const OrtGraph*) noexcept { return kCompatibility; }

// ---------------------------------------------------------------------------
// The factory.
struct Factory : OrtEpFactory {
  Api api;
  std::string name;
  std::mutex mu;
  std::unordered_map<const OrtHardwareDevice*, int> ordinals;  // hardware device -> CUDA ordinal
  std::vector<OrtMemoryInfo*> infos;                           // one per ordinal
  ~Factory() {
    for (OrtMemoryInfo* m : infos)
      if (m) api.ort->ReleaseMemoryInfo(m);
  }
  OrtMemoryInfo* memory_info(int ordinal) {
    std::lock_guard<std::mutex> lock(mu);
    if ((int)infos.size() <= ordinal) infos.resize(ordinal + 1, nullptr);
    if (infos[ordinal] == nullptr)
      api.ok(api.ort->CreateMemoryInfo_V2(kMemoryName, OrtMemoryInfoDeviceType_GPU, kNvidiaVendorId, ordinal,
                                          OrtDeviceMemoryType_DEFAULT, 256, OrtDeviceAllocator, &infos[ordinal]));
    return infos[ordinal];
  }
};

Factory& fself(OrtEpFactory* p) { return *static_cast<Factory*>(p); }
const Factory& fself(const OrtEpFactory* p) { return *static_cast<const Factory*>(p); }

const char* ORT_API_CALL f_name(const OrtEpFactory* p) noexcept { return fself(p).name.c_str(); }
const char* ORT_API_CALL f_vendor(const OrtEpFactory*) noexcept { return kVendor; }
uint32_t ORT_API_CALL f_vendor_id(const OrtEpFactory*) noexcept { return kNvidiaVendorId; }
const char* ORT_API_CALL f_version(const OrtEpFactory*) noexcept { return kVersion; }

// NVIDIA GPUs among ORT's hardware devices, numbered in the order ORT lists
// them (the CUDA ordinals when CUDA_DEVICE_ORDER=PCI_BUS_ID, ORT's order).
OrtStatus* ORT_API_CALL f_supported(OrtEpFactory* p, const OrtHardwareDevice* const* devs, size_t n,
                                    OrtEpDevice** out, size_t max_out, size_t* n_out) noexcept {
  Factory& f = fself(p);
  return guarded(f.api, [&] {
    if (n_out == nullptr) fail(ORT_INVALID_ARGUMENT, "requires a num_ep_devices output pointer");
    *n_out = 0;
    if (out)
      for (size_t i = 0; i < max_out; ++i) out[i] = nullptr;
    if (devs == nullptr || n == 0) return;
    if (f.api.ep == nullptr) fail(ORT_NOT_IMPLEMENTED, "requires OrtEpApi to create OrtEpDevice instances");
    int cuda_count = 0;
    if (cudaGetDeviceCount(&cuda_count) != cudaSuccess) {
      cudaGetLastError();
      cuda_count = 0;
    }
    int ordinal = 0;
    for (size_t i = 0; i < n && *n_out < max_out; ++i) {
      if (f.api.ort->HardwareDevice_Type(devs[i]) != OrtHardwareDeviceType_GPU ||
          f.api.ort->HardwareDevice_VendorId(devs[i]) != kNvidiaVendorId)
        continue;
      if (ordinal >= cuda_count) break;
      OrtEpDevice* d = nullptr;
      f.api.ok(f.api.ep->CreateEpDevice(p, devs[i], nullptr, nullptr, &d));
      f.api.ok(f.api.ep->EpDevice_AddAllocatorInfo(d, f.memory_info(ordinal)));
      {
        std::lock_guard<std::mutex> lock(f.mu);
        f.ordinals[devs[i]] = ordinal;
      }
      if (out) out[*n_out] = d;
      ++*n_out;
      ++ordinal;
    }
  });
}

OrtStatus* ORT_API_CALL f_create_ep(OrtEpFactory* p, const OrtHardwareDevice* const* devs, const OrtKeyValuePairs* const*,
                                    size_t n, const OrtSessionOptions*, const OrtLogger* logger, OrtEp** out) noexcept {
  Factory& f = fself(p);
  return guarded(f.api, [&] {
    if (out == nullptr) return;
    *out = nullptr;
    int ordinal = 0;
    if (devs && n) {
      std::lock_guard<std::mutex> lock(f.mu);
      auto it = f.ordinals.find(devs[0]);
      if (it != f.ordinals.end()) ordinal = it->second;
    }
    auto ep = std::make_unique<Ep>();
    std::memset(static_cast<OrtEp*>(ep.get()), 0, sizeof(OrtEp));
    ep->ort_version_supported = kApiFloor;
    ep->GetName = &ep_name;
    ep->GetCapability = &ep_get_capability;
    ep->Compile = &ep_compile;
    ep->ReleaseNodeComputeInfos = &ep_release_infos;
    ep->GetPreferredDataLayout = &ep_layout;
    ep->OnRunStart = &ep_run_start;
    ep->OnRunEnd = &ep_run_end;
    ep->GetCompiledModelCompatibilityInfo = &ep_compat;
    ep->api = f.api;
    if (logger) ep->api.logger = logger;
    ep->name = f.name;
    ep->device = ordinal;
    *out = ep.release();
  });
}

void ORT_API_CALL f_release_ep(OrtEpFactory*, OrtEp* ep) noexcept { delete static_cast<Ep*>(ep); }

OrtStatus* ORT_API_CALL f_validate(OrtEpFactory* p, const OrtHardwareDevice* const*, size_t, const char* info,
                                   OrtCompiledModelCompatibility* out) noexcept {
  Factory& f = fself(p);
  return guarded(f.api, [&] {
    if (out == nullptr) fail(ORT_INVALID_ARGUMENT, "requires a model_compatibility output pointer");
    *out = info && std::string_view(info) == kCompatibility ? OrtCompiledModelCompatibility_EP_SUPPORTED_OPTIMAL
                                                            : OrtCompiledModelCompatibility_EP_UNSUPPORTED;
  });
}

OrtStatus* ORT_API_CALL f_create_allocator(OrtEpFactory* p, const OrtMemoryInfo* mi, const OrtKeyValuePairs*,
                                           OrtAllocator** out) noexcept {
  Factory& f = fself(p);
  return guarded(f.api, [&] {
    if (out == nullptr) fail(ORT_INVALID_ARGUMENT, "requires an allocator output pointer");
    *out = nullptr;
    if (mi == nullptr || f.api.ep == nullptr) return;
    const OrtMemoryDevice* md = f.api.ep->MemoryInfo_GetMemoryDevice(mi);
    if (!our_device(f.api, md) || f.api.ep->MemoryDevice_GetMemoryType(md) != OrtDeviceMemoryType_DEFAULT)
      fail(ORT_INVALID_ARGUMENT, "CreateAllocator: only this EP's device memory is served");
    const int ordinal = (int)f.api.ep->MemoryDevice_GetDeviceId(md);
    auto a = std::make_unique<DeviceAllocator>();
    std::memset(static_cast<OrtAllocator*>(a.get()), 0, sizeof(OrtAllocator));
    a->version = ORT_API_VERSION;
    a->Alloc = &alloc_impl;
    a->Free = &free_impl;
    a->Info = &info_impl;
    a->Reserve = &alloc_impl;
    a->GetStats = &stats_impl;
    a->api = &f.api;
    a->info = f.memory_info(ordinal);
    a->device = ordinal;
    *out = a.release();
  });
}

void ORT_API_CALL f_release_allocator(OrtEpFactory*, OrtAllocator* a) noexcept { delete static_cast<DeviceAllocator*>(a); }

OrtStatus* ORT_API_CALL f_data_transfer(OrtEpFactory* p, OrtDataTransferImpl** out) noexcept {
  Factory& f = fself(p);
  return guarded(f.api, [&] {
    if (out == nullptr) fail(ORT_INVALID_ARGUMENT, "requires a data_transfer output pointer");
    auto t = std::make_unique<Transfer>();
    std::memset(static_cast<OrtDataTransferImpl*>(t.get()), 0, sizeof(OrtDataTransferImpl));
    t->ort_version_supported = ORT_API_VERSION;
    t->Release = &transfer_release;
    t->CanCopy = &transfer_can_copy;
    t->CopyTensors = &transfer_copy;
    t->api = &f.api;
    *out = t.release();
  });
}

bool ORT_API_CALL f_stream_aware(const OrtEpFactory*) noexcept { return true; }

OrtStatus* ORT_API_CALL f_create_stream(OrtEpFactory* p, const OrtMemoryDevice* md, const OrtKeyValuePairs*,
                                        OrtSyncStreamImpl** out) noexcept {
  Factory& f = fself(p);
  return guarded(f.api, [&] {
    if (out == nullptr) fail(ORT_INVALID_ARGUMENT, "requires a stream output pointer");
    *out = nullptr;
    if (md == nullptr || !our_device(f.api, md)) return;
    *out = make_stream(&f.api, (int)f.api.ep->MemoryDevice_GetDeviceId(md));
  });
}

OrtStatus* ORT_API_CALL f_incompat(OrtEpFactory*, const OrtHardwareDevice*, OrtDeviceEpIncompatibilityDetails*) noexcept {
  return nullptr;
}
OrtStatus* ORT_API_CALL f_importer(OrtEpFactory*, const OrtEpDevice*, OrtExternalResourceImporterImpl** out) noexcept {
  if (out) *out = nullptr;
  return nullptr;
}
OrtStatus* ORT_API_CALL f_num_domains(OrtEpFactory*, size_t* n) noexcept {
  if (n) *n = 0;
  return nullptr;
}
OrtStatus* ORT_API_CALL f_domains(OrtEpFactory*, OrtCustomOpDomain**, size_t) noexcept { return nullptr; }
OrtStatus* ORT_API_CALL f_interop(OrtEpFactory* p, const OrtEpDevice*, const OrtGraphicsInteropConfig*) noexcept {
  Factory& f = fself(p);
  return f.api.ort ? f.api.ort->CreateStatus(ORT_NOT_IMPLEMENTED, "Doe ORT plugin EP: no graphics interop") : nullptr;
}
OrtStatus* ORT_API_CALL f_deinterop(OrtEpFactory*, const OrtEpDevice*) noexcept { return nullptr; }

}  // namespace doeep

using namespace doeep;

DOE_EP_EXPORT OrtStatus* CreateEpFactories(const char* registered_name, const OrtApiBase* api_base,
                                           const OrtLogger* logger, OrtEpFactory** factories,
                                           size_t max_factories, size_t* num_factories) {
  Api api;
  api.base = api_base;
  api.ort = api_base ? api_base->GetApi(kApiFloor) : nullptr;
  api.ep = api.ort ? api.ort->GetEpApi() : nullptr;
  api.logger = logger;
  if (num_factories) *num_factories = 0;
  return guarded(api, [&] {
    if (factories == nullptr || num_factories == nullptr)
      fail(ORT_INVALID_ARGUMENT, "requires factories and num_factories output pointers");
    if (max_factories < 1) fail(ORT_INVALID_ARGUMENT, "requires space for at least one factory");
    if (api.ort == nullptr) fail(ORT_FAIL, "the ORT API at version 23 is unavailable");
    auto f = std::make_unique<Factory>();
    std::memset(static_cast<OrtEpFactory*>(f.get()), 0, sizeof(OrtEpFactory));
    f->ort_version_supported = kApiFloor;
    f->GetName = &f_name;
    f->GetVendor = &f_vendor;
    f->GetSupportedDevices = &f_supported;
    f->CreateEp = &f_create_ep;
    f->ReleaseEp = &f_release_ep;
    f->GetVendorId = &f_vendor_id;
    f->GetVersion = &f_version;
    f->ValidateCompiledModelCompatibilityInfo = &f_validate;
    f->CreateAllocator = &f_create_allocator;
    f->ReleaseAllocator = &f_release_allocator;
    f->CreateDataTransfer = &f_data_transfer;
    f->IsStreamAware = &f_stream_aware;
    f->CreateSyncStreamForDevice = &f_create_stream;
    f->GetHardwareDeviceIncompatibilityDetails = &f_incompat;
    f->CreateExternalResourceImporterForDevice = &f_importer;
    f->GetNumCustomOpDomains = &f_num_domains;
    f->GetCustomOpDomains = &f_domains;
    f->InitGraphicsInterop = &f_interop;
    f->DeinitGraphicsInterop = &f_deinterop;
    f->api = api;
    f->name = registered_name && registered_name[0] ? registered_name : kDefaultName;
    factories[0] = f.release();
    *num_factories = 1;
  });
}

DOE_EP_EXPORT OrtStatus* ReleaseEpFactory(OrtEpFactory* factory) {
  delete static_cast<Factory*>(factory);
  return nullptr;
}

DOE_EP_EXPORT void DoeOrtEpResetDebugCounters() {
  for (auto& c : g_counters) c.store(0, std::memory_order_relaxed);
  g_decoder_claimed.store(0);
  g_decoder_computed.store(0);
}

DOE_EP_EXPORT void DoeOrtEpGetDebugCounters(doeep::DebugCounters* out) {
  if (out == nullptr) return;
  uint64_t* dst = reinterpret_cast<uint64_t*>(out);
  for (size_t i = 0; i < kNumCounters; ++i) dst[i] = g_counters[i].load(std::memory_order_relaxed);
}

// Claimed nodes and Compute calls of the decoder-block kinds (no reference field).
DOE_EP_EXPORT void DoeOrtEpGetDecoderCounters(uint64_t* claimed, uint64_t* computed) {
  if (claimed) *claimed = g_decoder_claimed.load();
  if (computed) *computed = g_decoder_computed.load();
}
