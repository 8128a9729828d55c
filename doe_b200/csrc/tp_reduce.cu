// tp_reduce.cu -- the decoder block's tensor-parallel AllReduce, fused into
// the RMSNorm that consumes it, over peer buffers mapped with CUDA IPC.
//
// Each rank's linear layer writes its partial product (rank 0's with the
// residual added) into a slot of its own peer buffer.  One launch per rank
// then publishes "my slot is complete" to every peer (a system-scope release
// store into the peer's flag for this rank), waits for the peers' flags
// (system-scope acquire loads of its own flags, bounded), and sums the world
// partials of each row in rank order with loads over NVLink, so every rank
// computes bit-identical sums.  It stores the sums (the residual stream) and,
// with gamma, the normalised bf16 row, as doe_rmsnorm_bf16 does.  The grid
// is one CTA per row.  The call's epoch is a counter in the buffer that the
// last CTA of each launch advances, so a CUDA graph replays it unchanged.
#include "common.cuh"

namespace doe {
namespace tp {

constexpr uint32_t OFF_FLAGS = 0;   // u64 [DOE_TP_MAX_RANKS], written by the peers
constexpr uint32_t OFF_EPOCH = 64;  // u64, this rank's last completed epoch
constexpr uint32_t OFF_EXIT = 72;   // u32, CTAs of the running launch that finished
constexpr uint32_t OFF_SLOTS = 256;
constexpr int kThreads = 1024;  // a 4096-wide row: one 16-byte column group per thread, every
                                // peer's load of it in flight at once
constexpr long long kWaitCycles = 4000000000LL;  // ~2 s at 1.9 GHz

struct Args {
  uint8_t* buf[DOE_TP_MAX_RANKS];
  int rank, world, slot, rows, cols;
  const __nv_bfloat16* gamma;
  float eps;
  float* h_out;
  __nv_bfloat16* xn_out;
  int32_t* status;
};

__device__ __forceinline__ void st_release_sys(uint64_t* p, uint64_t v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;\n" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_acquire_sys(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];\n" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__global__ void __launch_bounds__(kThreads) reduce_rmsnorm_kernel(const Args a) {
  __shared__ float warp_sum[kThreads / 32];
  pdl_wait();  // this rank's partial (the previous kernel's output) is complete
  pdl_trigger();
  uint8_t* own = a.buf[a.rank];
  const uint64_t epoch = *reinterpret_cast<volatile uint64_t*>(own + OFF_EPOCH) + 1;
  const int t = threadIdx.x;
  if (blockIdx.x == 0 && t < a.world && t != a.rank)
    st_release_sys(reinterpret_cast<uint64_t*>(a.buf[t] + OFF_FLAGS) + a.rank, epoch);
  if (t < a.world && t != a.rank) {
    const uint64_t* f = reinterpret_cast<const uint64_t*>(own + OFF_FLAGS) + t;
    if (ld_acquire_sys(f) < epoch) {
      const long long t0 = clock64();
      while (ld_acquire_sys(f) < epoch) {
        if (clock64() - t0 > kWaitCycles) {
          // the sums below then read whatever the peer's slot holds; the
          // status word tells the host
          report(a.status, DOE_DEVICE_ERR_TIMEOUT);
          break;
        }
        __nanosleep(128);
      }
    }
  }
  __syncthreads();

  const size_t row_off = (size_t)a.slot * a.rows * a.cols + (size_t)blockIdx.x * a.cols;
  const int n4 = a.cols >> 2;
  float4* h4 = reinterpret_cast<float4*>(a.h_out + (size_t)blockIdx.x * a.cols);
  float ss = 0.0f;
  for (int i = t; i < n4; i += kThreads) {
    float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    for (int r = 0; r < a.world; ++r) {
      const float4* src =
          reinterpret_cast<const float4*>(reinterpret_cast<const float*>(a.buf[r] + OFF_SLOTS) + row_off) + i;
      // a peer's slot is read past every cache (it changes between epochs)
      const float4 v = r == a.rank ? *src : __ldcv(src);
      acc.x += v.x;
      acc.y += v.y;
      acc.z += v.z;
      acc.w += v.w;
    }
    h4[i] = acc;
    ss += acc.x * acc.x + acc.y * acc.y + acc.z * acc.z + acc.w * acc.w;
  }
  if (a.gamma != nullptr) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((t & 31) == 0) warp_sum[t >> 5] = ss;
    __syncthreads();
    float total = 0.0f;
#pragma unroll
    for (int w = 0; w < kThreads / 32; ++w) total += warp_sum[w];
    const float inv = 1.0f / sqrtf(total / (float)a.cols + a.eps);
    const uint2* g2 = reinterpret_cast<const uint2*>(a.gamma);
    uint2* o2 = reinterpret_cast<uint2*>(a.xn_out + (size_t)blockIdx.x * a.cols);
    for (int i = t; i < n4; i += kThreads) {
      const float4 v = h4[i];  // written above by this thread
      const uint2 gw = g2[i];
      const float2 g01 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&gw.x));
      const float2 g23 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&gw.y));
      __nv_bfloat162 y01 = __floats2bfloat162_rn(v.x * inv * g01.x, v.y * inv * g01.y);
      __nv_bfloat162 y23 = __floats2bfloat162_rn(v.z * inv * g23.x, v.w * inv * g23.y);
      uint2 ow;
      ow.x = *reinterpret_cast<uint32_t*>(&y01);
      ow.y = *reinterpret_cast<uint32_t*>(&y23);
      o2[i] = ow;
    }
  }
  // the last CTA of the launch advances the epoch (every CTA read it above)
  __syncthreads();
  if (t == 0) {
    unsigned* exit_ctr = reinterpret_cast<unsigned*>(own + OFF_EXIT);
    __threadfence();
    if (atomicAdd(exit_ctr, 1u) == gridDim.x - 1) {
      *exit_ctr = 0u;
      *reinterpret_cast<volatile uint64_t*>(own + OFF_EPOCH) = epoch;
    }
  }
}

}  // namespace tp

uint64_t tp_buffer_bytes(uint32_t rows, uint32_t cols) {
  return tp::OFF_SLOTS + 2ull * rows * cols * sizeof(float);
}

float* tp_slot_ptr(void* buffer, uint32_t slot, uint32_t rows, uint32_t cols) {
  return reinterpret_cast<float*>(static_cast<uint8_t*>(buffer) + tp::OFF_SLOTS) + (size_t)slot * rows * cols;
}

int launch_tp_reduce_rmsnorm(const doe_tp_peers* p, uint32_t slot, const void* gamma, float eps, float* h_out,
                             void* xn_out, uint32_t rows, uint32_t cols, const doe_launch* launch) {
  tp::Args a;
  for (int i = 0; i < DOE_TP_MAX_RANKS; ++i)
    a.buf[i] = i < (int)p->world ? static_cast<uint8_t*>(p->buffers[i]) : nullptr;
  a.rank = (int)p->rank;
  a.world = (int)p->world;
  a.slot = (int)slot;
  a.rows = (int)rows;
  a.cols = (int)cols;
  a.gamma = static_cast<const __nv_bfloat16*>(gamma);
  a.eps = eps;
  a.h_out = h_out;
  a.xn_out = static_cast<__nv_bfloat16*>(xn_out);
  a.status = launch->status;
  return cuda_status(launch_pdl(tp::reduce_rmsnorm_kernel, dim3(rows), dim3(tp::kThreads), 0,
                                static_cast<cudaStream_t>(launch->stream), a),
                     "reduce_rmsnorm_kernel");
}

}  // namespace doe
