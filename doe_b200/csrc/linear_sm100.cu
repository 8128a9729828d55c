// linear_sm100.cu -- the decoder block's matrix products and RMSNorm for
// decode-sized batches on sm_100a.
//
// y[b, n] = sum_k x[b, k] w[n, k] with batch <= 32 is a weight stream: each
// weight byte is read once and used for at most 32 products, so the product
// is HBM-bound and the kernel's job is to keep every SM's share of the weight
// bytes in flight.  The product is turned around so the weights are the MMA's
// M side: D[128 weight rows, 32 batch] += W[128 x 16] * X^T[16 x 32] with
// tcgen05.mma kind::f16 (bf16 operands, f32 accumulation in TMEM).
//
// Work split (stream-K): the (tile, 64-wide k block) iterations of the whole
// product are divided evenly over a persistent grid of at most one CTA per
// SM, so the grid is balanced for any (n_out, k); a CTA's range can start and
// end inside a tile.  A CTA that covers a whole tile runs the epilogue from
// TMEM.  A split tile is finished by the CTA holding its first k block, for
// which it is the last segment: the later contributors (for which it is the
// first) write their f32 partial tiles to the workspace and count in, and the
// finisher waits for the count, adds the partials to its own accumulator in
// contributor order (the result does not depend on timing) and runs the
// epilogue.  That wait needs every CTA of the grid resident at once, which a
// grid of at most one CTA per SM gives; it is bounded like every other wait.
// Work split (cluster): when there are at most half as many tiles as SMs, a
// tile's k range is split over a cluster of up to 4 CTAs instead (the largest
// size whose clusters are all resident at once).  Ranks 1-3 send their f32
// accumulators into rank 0's shared memory with st.async over distributed
// shared memory; rank 0 sums them in rank order and runs the epilogue.
// Epilogues: store into up to three column segments (bf16, f16 or f32),
// SwiGLU over interleaved 64-row gate / up blocks, or f32 plus a residual.
// Results leave through shared memory, transposed so that each lane writes
// one batch row's columns with 16-byte stores.  A split RMSNorm
// (doe_linear_norm): the f32 producer also writes bf16(y * gamma) and each
// row's sum of squares per 32 columns; a consumer scales its rows by
// 1 / sqrt(mean + eps) from those sums before its epilogue.
// Launched with programmatic dependent launch: the first ring of weight
// boxes is issued before griddepcontrol.wait, since no kernel of a step
// writes the weights.
//
//   warp 0     TMA producer: per k block one 128 x 64 weight box and one
//              32 x 64 activation box (rows past `batch` read as zero) into
//              an 8-stage ring, 128-byte swizzle
//   warp 1     TMEM owner + MMA issuer (one elected lane): 4 MMAs of K = 16
//              per stage into one of two 32-column accumulators, so the
//              epilogue of one tile overlaps the MMAs of the next
//   warps 2-5  epilogue: warp w reads TMEM lane quarter w % 4 (32 weight
//              rows), 32 batch columns per thread
//
// Every mbarrier wait is bounded; on timeout the kernel sets
// DOE_DEVICE_ERR_TIMEOUT, the roles stop, copies and MMAs still in flight are
// waited for (bounded) and TMEM is freed.  No cluster multicast.
#include <atomic>

#include <cuda.h>
#include <cudaTypedefs.h>

#include "tma.cuh"
#include "umma.cuh"

namespace doe {
namespace lin {

constexpr int BM = 128, NB = 32;
constexpr int kBoxes = 1;                 // 64-wide k boxes per stage
constexpr int BK = 64 * kBoxes;           // k per stage
constexpr int kStages = 8;
constexpr int kMinIters = 2;              // fewest stages a CTA streams
constexpr int kMaxSplit = 8;              // most CTAs sharing one tile
constexpr int kCtasPerSm = 1;
constexpr uint32_t kWBox = BM * 64 * 2;   // 16 KB: 128 weight rows x 64 k
constexpr uint32_t kXBox = NB * 64 * 2;   // 4 KB: 32 activation rows x 64 k
constexpr uint32_t kWBytes = kBoxes * kWBox;
constexpr uint32_t kXBytes = kBoxes * kXBox;
constexpr uint32_t kStageBytes = kWBytes + kXBytes;  // a multiple of 1024
constexpr int kThreads = 192;
constexpr uint32_t kTmemCols = 2 * NB;
constexpr int kMaxCtas = 512;
constexpr long long kWaitCycles = 4000000000LL;  // ~2 s at 1.9 GHz

constexpr int kMaxCluster = 4;            // CTAs of one tile in cluster mode
enum Bar { FULL0 = 0, EMPTY0 = FULL0 + kStages, ACC_FULL0 = EMPTY0 + kStages, ACC_EMPTY0 = ACC_FULL0 + 2,
           MMA_DONE = ACC_EMPTY0 + 2, RECV_FULL = MMA_DONE + 1, NUM_BARS };
constexpr uint32_t OFF_BAR = kStages * kStageBytes;
constexpr uint32_t OFF_MISC = OFF_BAR + 8 * NUM_BARS;  // TMEM slot, abort flag
constexpr uint32_t OFF_RSCALE = OFF_MISC + 64;          // consumer's row scales [NB] f32
constexpr uint32_t OFF_XCHG = OFF_BAR + 512;            // SwiGLU mate values [NB / 2][128] f32
static_assert(OFF_RSCALE + NB * 4 <= OFF_XCHG, "misc area");
constexpr uint32_t kTileBytes = BM * NB * 4;            // one f32 accumulator tile (16 KB)
// cluster mode: the other CTAs' accumulator tiles, row r's 32 values in one
// 128-byte line with 16-byte chunk c at c ^ (r & 7)
constexpr uint32_t OFF_RECV = ((OFF_XCHG + NB * 64 * 4 + 1023) / 1024) * 1024;
constexpr uint32_t kSmemBytes = OFF_RECV + (kMaxCluster - 1) * kTileBytes + 1024;  // + alignment slack

struct Args {
  void* out[3];
  int seg_end[3];          // exclusive end (output column) of each segment
  const float* residual;   // [batch, n_out] f32 or null
  float* part;             // [ctas][2][NB][BM] f32 partial tiles
  unsigned* counters;      // [tiles], zero between launches
  int32_t* status;
  int batch, n_out, kb, tiles, ctas, epilogue, dtype;
  long long iters;         // tiles * kb
  int cluster;             // > 1: cluster mode, this many CTAs per tile; else stream-K
  // RMSNorm split over two products (doe_linear_norm): the producer of the
  // residual stream also writes bf16(y * gamma) and per-32-column sums of
  // squares; the consumer scales its rows by 1 / sqrt(sum / k + eps)
  const __nv_bfloat16* gamma_out;  // [n_out] or null
  __nv_bfloat16* normed_out;       // [batch, n_out]
  float* ssq_out;                  // [n_out / 32][NB]
  const float* ssq_in;             // [k / 32][NB] or null
  float eps;
};

__device__ __forceinline__ bool wait_bar(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                         int32_t* status) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if (clock64() - t0 > kWaitCycles) {
      *abort_flag = 1;
      report(status, DOE_DEVICE_ERR_TIMEOUT);
      return false;
    }
  }
}

// The four epilogue warps (128 threads) on named barrier 1.
__device__ __forceinline__ void epi_sync() { asm volatile("bar.sync 1, 128;\n" ::: "memory"); }
__device__ __forceinline__ bool epi_all(bool ok) {
  uint32_t r;
  asm volatile(
      "{\n.reg .pred p, q;\nsetp.ne.u32 p, %1, 0;\nbar.red.and.pred q, 1, 128, p;\nselp.u32 %0, 1, 0, q;\n}\n"
      : "=r"(r)
      : "r"((uint32_t)ok)
      : "memory");
  return r != 0;
}

// Cluster mode: the rank that finishes row block q (rows 32q .. 32q + 31) of
// the tile.  The blocks are dealt round the cluster so every rank sums and
// stores a share; SwiGLU pairs row r with r + 64, so rank 0 keeps them all.
__device__ __forceinline__ int block_owner(int q, const Args& a) {
  return a.epilogue == DOE_LINEAR_SWIGLU ? 0 : q % a.cluster;
}
// Bytes the other ranks send to `rank`: each owned row, once from each of them.
__device__ __forceinline__ uint32_t recv_bytes(int rank, const Args& a) {
  uint32_t n = 0;
  for (int q = 0; q < 4; ++q) n += block_owner(q, a) == rank ? 32u : 0u;
  return n * (uint32_t)(a.cluster - 1) * (NB * 4);
}

__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ long long it_begin(long long c, const Args& a) { return c * a.iters / a.ctas; }

// This CTA's (tile, k block) iterations [it0, it1): in cluster mode rank r of
// the tile's cluster takes the r-th of a.cluster even k ranges; otherwise the
// stream-K share.
__device__ __forceinline__ void cta_range(const Args& a, long long& it0, long long& it1) {
  if (a.cluster > 1) {
    const long long tile = blockIdx.x / a.cluster, r = blockIdx.x % a.cluster;
    it0 = tile * a.kb + r * a.kb / a.cluster;
    it1 = tile * a.kb + (r + 1) * a.kb / a.cluster;
  } else {
    it0 = it_begin(blockIdx.x, a);
    it1 = it_begin(blockIdx.x + 1, a);
  }
}

// Distributed shared memory: `addr` of this CTA's window -> the same offset in
// cluster CTA `rank`.
__device__ __forceinline__ uint32_t mapa_rank(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;\n" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
// 16 bytes into another cluster CTA's shared memory, counted on its mbarrier.
__device__ __forceinline__ void st_async_v4(uint32_t addr, float x, float y, float z, float w, uint32_t bar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.f32 [%0], {%1, %2, %3, %4}, [%5];\n" ::"r"(
                   addr),
               "f"(x), "f"(y), "f"(z), "f"(w), "r"(bar)
               : "memory");
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;\n" ::: "memory");
}
// The CTA whose iteration range holds iteration i.
__device__ __forceinline__ int cta_of(long long i, const Args& a) {
  return (int)(((i + 1) * a.ctas - 1) / a.iters);
}

// eight f32 values as eight bf16 (or f16), rounded to nearest even
__device__ __forceinline__ uint4 pack8(const float* y, bool bf16) {
  uint32_t w[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    if (bf16) {
      const __nv_bfloat162 h = __floats2bfloat162_rn(y[2 * e], y[2 * e + 1]);
      w[e] = *reinterpret_cast<const uint32_t*>(&h);
    } else {
      const __half2 h = __floats2half2_rn(y[2 * e], y[2 * e + 1]);
      w[e] = *reinterpret_cast<const uint32_t*>(&h);
    }
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

__global__ void __launch_bounds__(kThreads, kCtasPerSm)
    linear_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_x,
                  const Args a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_addr(smem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + OFF_MISC + 8);
  float* xchg = reinterpret_cast<float*>(smem + OFF_XCHG);
  auto bar = [&](int i) { return smem_addr(&bars[i]); };

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  long long it0, it1;
  cta_range(a, it0, it1);
  const uint32_t crank = a.cluster > 1 ? blockIdx.x % a.cluster : 0;  // rank in the tile's cluster

  if (threadIdx.x == 0) {
    for (int i = 0; i < NUM_BARS; ++i) mbar_init(bar(i), (i >= ACC_EMPTY0 && i < ACC_EMPTY0 + 2) ? 4u : 1u);
    *abort_flag = 0;
    // cluster mode: the tile's other CTAs send their accumulators here
    if (a.cluster > 1 && recv_bytes((int)crank, a) > 0) mbar_expect_tx(bar(RECV_FULL), recv_bytes((int)crank, a));
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(
                     smem_addr(tmem_slot)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::);
  }
  tc_fence_before();
  __syncthreads();
  if (a.cluster > 1) cluster_sync_all();  // every CTA's barriers exist before any remote store
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_trigger();

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      // The weights are never written by a kernel of the step: the first ring
      // of weight boxes is issued before waiting for the previous kernel (the
      // producer of x), whose tail it overlaps.
      const long long npre = min((long long)kStages, it1 - it0);
      for (long long j = 0; j < npre; ++j) {
        const long long it = it0 + j;
        const int tile = (int)(it / a.kb), k = (int)(it - (long long)tile * a.kb);
        const uint32_t dst = sbase + (uint32_t)j * kStageBytes;
        mbar_expect_tx(bar(FULL0 + (int)j), kStageBytes);
#pragma unroll
        for (int b = 0; b < kBoxes; ++b)
          tma_load_3d(dst + b * kWBox, &tm_w, bar(FULL0 + (int)j), k * BK + b * 64, 0, tile * BM);
      }
      pdl_wait();
      for (long long j = 0; j < npre; ++j) {
        const long long it = it0 + j;
        const int k = (int)(it - (it / a.kb) * a.kb);
        const uint32_t dst = sbase + (uint32_t)j * kStageBytes;
#pragma unroll
        for (int b = 0; b < kBoxes; ++b)
          tma_load_3d(dst + kWBytes + b * kXBox, &tm_x, bar(FULL0 + (int)j), k * BK + b * 64, 0, 0);
      }
      long long n = npre;
      bool ok = true;
      for (long long it = it0 + npre; it < it1; ++it, ++n) {
        const int s = (int)(n % kStages);
        if (n >= kStages && !(ok = wait_bar(bar(EMPTY0 + s), (uint32_t)((n / kStages) - 1) & 1, abort_flag,
                                            a.status)))
          break;
        const int tile = (int)(it / a.kb), k = (int)(it - (long long)tile * a.kb);
        const uint32_t dst = sbase + s * kStageBytes;
        mbar_expect_tx(bar(FULL0 + s), kStageBytes);
#pragma unroll
        for (int b = 0; b < kBoxes; ++b) {
          tma_load_3d(dst + b * kWBox, &tm_w, bar(FULL0 + s), k * BK + b * 64, 0, tile * BM);
          tma_load_3d(dst + kWBytes + b * kXBox, &tm_x, bar(FULL0 + s), k * BK + b * 64, 0, 0);
        }
      }
      if (!ok) {
        // no copy may land after the CTA exits: wait for the last issued ones
        for (long long j = n > kStages ? n - kStages : 0; j < n; ++j)
          mbar_wait_bounded(bar(FULL0 + (int)(j % kStages)), (uint32_t)(j / kStages) & 1);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    const uint32_t idesc = idesc_kind_f16(true, false, BM, NB);
    const uint64_t d0 = sdesc(sbase, 16, 1024);  // stage 0's weight box; its activations kWBytes on
    auto wait = [&](int b, uint32_t parity) {
      return __all_sync(0xffffffffu, wait_bar(bar(b), parity, abort_flag, a.status));
    };
    long long n = 0;
    int seg = 0;
    bool ok = true;
    for (long long it = it0; it < it1 && ok; ++seg) {
      const long long tile = it / a.kb;
      const long long end = min(it1, (tile + 1) * a.kb);
      const int acc = seg & 1;
      if (seg >= 2 && !(ok = wait(ACC_EMPTY0 + acc, (uint32_t)((seg >> 1) - 1) & 1))) break;
      tc_fence_after();
      const long long first = it;
      for (; it < end; ++it, ++n) {
        const int s = (int)(n % kStages);
        if (!(ok = wait(FULL0 + s, (uint32_t)(n / kStages) & 1))) break;
        tc_fence_after();
        const uint64_t dw = d0 + ((s * kStageBytes) >> 4), dx = d0 + ((s * kStageBytes + kWBytes) >> 4);
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk)
          umma_elect(tmem + acc * NB, dw + (((kk >> 2) * kWBox + (kk & 3) * 32) >> 4),
                     dx + (((kk >> 2) * kXBox + (kk & 3) * 32) >> 4), idesc, (it > first || kk > 0) ? 1u : 0u);
        commit_elect(bar(EMPTY0 + s));  // the stage is free once these MMAs are done
      }
      if (ok) commit_elect(bar(ACC_FULL0 + acc));
    }
    // every MMA this warp issued has finished once MMA_DONE flips
    commit_elect(bar(MMA_DONE));
    __all_sync(0xffffffffu, mbar_wait_bounded(bar(MMA_DONE), 0));
  } else {
    // ------------------------------------------------------------ epilogue
    pdl_wait();  // residual, outputs and the workspace belong to earlier kernels until then
    const int q = warp & 3;
    const int row = q * 32 + lane;  // weight row within the tile = TMEM lane
    const uint32_t t_lane = tmem + ((uint32_t)(q * 32) << 16);
    const float* rscale = reinterpret_cast<const float*>(smem + OFF_RSCALE);
    if (a.ssq_in != nullptr) {
      // consumer of a split RMSNorm: batch row b's sum of squares over the
      // k / 32 column blocks, thread (b, part) adding blocks part, part + 4,
      // ... in order, then the four parts pairwise; computed while the MMAs run
      const int b = row >> 2, part = row & 3;
      const int nblk = a.kb * (BK / 32);
      float sum = 0.0f;
#pragma unroll 8
      for (int i = part; i < nblk; i += 4) sum += a.ssq_in[(size_t)i * NB + b];
      sum += __shfl_xor_sync(0xffffffffu, sum, 1);
      sum += __shfl_xor_sync(0xffffffffu, sum, 2);
      if (part == 0)
        reinterpret_cast<float*>(smem + OFF_RSCALE)[b] = 1.0f / sqrtf(sum / (float)(a.kb * BK) + a.eps);
      epi_sync();
    }
    int seg = 0;
    for (long long it = it0; it < it1; ++seg) {
      const long long tile = it / a.kb;
      const long long end = min(it1, (tile + 1) * a.kb);
      const bool whole = it == tile * a.kb && end == (tile + 1) * a.kb;
      it = end;
      const int acc = seg & 1;
      // a residual this CTA will certainly add (a whole tile, or the tile of a
      // cluster's rank 0) is loaded while the MMAs still run, so its latency
      // leaves the tail of the launch
      const bool pre_res = a.residual != nullptr && a.epilogue != DOE_LINEAR_SWIGLU &&
                           (whole || (a.cluster > 1 && block_owner(q, a) == (int)crank));
      // the norm producer's gamma for the warp's 32 columns (64 bytes), copied
      // into the warp's 64 bytes of the exchange area (unused without SwiGLU)
      // while the MMAs run
      const uint32_t gsm = sbase + OFF_XCHG + (uint32_t)q * 64;
      if (a.normed_out != nullptr && lane < 4)
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\ncp.async.commit_group;\n" ::"r"(gsm + lane * 16),
                     "l"(a.gamma_out + (size_t)tile * BM + q * 32 + lane * 8)
                     : "memory");
      float rres[NB];
      if (pre_res) {
        const size_t col = (size_t)tile * BM + row;
#pragma unroll
        for (int j = 0; j < NB; ++j) rres[j] = j < a.batch ? a.residual[(size_t)j * a.n_out + col] : 0.0f;
      }
      const bool ok = epi_all(wait_bar(bar(ACC_FULL0 + acc), (uint32_t)(seg >> 1) & 1, abort_flag, a.status));
      if (!ok) break;
      tc_fence_after();
      uint32_t r[NB];
      tmem_ld32(t_lane + acc * NB, r);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(ACC_EMPTY0 + acc));
      float v[NB];
#pragma unroll
      for (int j = 0; j < NB; ++j) v[j] = __uint_as_float(r[j]);

      if (a.cluster > 1) {
        // the tile's k ranges were split over a cluster: each row block is
        // finished by its owner rank; the other ranks send it their rows into
        // the owner's shared memory (slot = sender rank, skipping the owner)
        // and the owner adds them to its own in that fixed order
        const uint32_t line = (uint32_t)row * 128u;
        const int own = block_owner(q, a);
        if (own != (int)crank) {
          const int slot = (int)crank < own ? (int)crank : (int)crank - 1;
          const uint32_t dst = mapa_rank(sbase + OFF_RECV + slot * kTileBytes + line, (uint32_t)own);
          const uint32_t rbar = mapa_rank(bar(RECV_FULL), (uint32_t)own);
#pragma unroll
          for (int c = 0; c < NB / 4; ++c)
            st_async_v4(dst + (((uint32_t)c ^ (row & 7)) << 4), v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3],
                        rbar);
          continue;
        }
        if (!__all_sync(0xffffffffu, wait_bar(bar(RECV_FULL), 0, abort_flag, a.status))) break;
        for (int slot = 0; slot < a.cluster - 1; ++slot) {
          const uint8_t* rl = smem + OFF_RECV + slot * kTileBytes + line;
#pragma unroll
          for (int c = 0; c < NB / 4; ++c) {
            const float4 t = *reinterpret_cast<const float4*>(rl + ((c ^ (row & 7)) << 4));
            v[4 * c] += t.x;
            v[4 * c + 1] += t.y;
            v[4 * c + 2] += t.z;
            v[4 * c + 3] += t.w;
          }
        }
      } else if (!whole) {
        // Stream-K fix-up.  The tile's k blocks run on CTAs c0..c1 in order.
        // For c0, which holds k block 0, the tile is its last segment; for
        // every later contributor it is the first, so they finish their share
        // early.  They store their f32 partial tile and count in; c0 waits
        // (bounded) for the count, adds the partials to its own accumulator
        // in contributor order (the sum c0 + c0+1 + ... of before) and runs
        // the epilogue, with no round trip of its own partial through memory.
        const int c0 = cta_of(tile * a.kb, a), c1 = cta_of((tile + 1) * a.kb - 1, a);
        if ((int)blockIdx.x != c0) {
          float* p = a.part + ((size_t)blockIdx.x * 2) * NB * BM + row;  // slot 0: this CTA's first tile
#pragma unroll
          for (int j = 0; j < NB; ++j) __stcg(p + j * BM, v[j]);
          __threadfence();
          epi_sync();
          if (threadIdx.x == 64) atomicAdd(&a.counters[tile], 1u);
          continue;
        }
        if (threadIdx.x == 64) {
          const unsigned want = (unsigned)(c1 - c0);
          const long long t0 = clock64();
          while (ld_acquire_u32(&a.counters[tile]) < want) {
            if (clock64() - t0 > kWaitCycles) {
              *abort_flag = 1;
              report(a.status, DOE_DEVICE_ERR_TIMEOUT);
              break;
            }
            __nanosleep(64);
          }
          a.counters[tile] = 0u;  // ready for the next launch
        }
        epi_sync();
        if (*abort_flag) break;
        __threadfence();
        // the later contributors in order, four partial tiles in flight at a time
        for (int c = c0 + 1; c <= c1; c += 4) {
          float t[4][NB];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            if (c + u <= c1) {
              const float* pc = a.part + ((size_t)(c + u) * 2) * NB * BM + row;
#pragma unroll
              for (int j = 0; j < NB; ++j) t[u][j] = __ldcg(pc + j * BM);
            }
          }
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            if (c + u <= c1) {
#pragma unroll
              for (int j = 0; j < NB; ++j) v[j] += t[u][j];
            }
          }
        }
      }

      if (a.ssq_in != nullptr) {
#pragma unroll
        for (int j = 0; j < NB; ++j) v[j] *= rscale[j];
      }

      if (a.epilogue == DOE_LINEAR_SWIGLU) {
        // rows 0-63 of the tile are gate rows, 64-127 the matching up rows;
        // the threads of rows r and r + 64 split the batch: the gate-row
        // thread finishes columns [0, 16), the up-row thread [16, 32), each
        // taking its mate's value for those columns through shared memory,
        // so all four epilogue warps share the SwiGLU (one warp per
        // scheduler, with the exponentials on the SFU)
        const bool gate = row < 64;
        const int j0 = gate ? 0 : NB / 2;
#pragma unroll
        for (int jj = 0; jj < NB / 2; ++jj) xchg[jj * 128 + row] = gate ? v[NB / 2 + jj] : v[jj];
        epi_sync();
        const size_t width = (size_t)a.n_out / 2;
        const int mate = row ^ 64;
        // the (feature, batch row) results go through shared memory (the
        // receive area, free once every epilogue warp has passed the barrier
        // above; rows padded to 68 floats) so that warp q stores features
        // [16 q, 16 q + 16) of batch row `lane` with 16-byte stores
        float* ty = reinterpret_cast<float*>(smem + OFF_RECV);
#pragma unroll
        for (int jj = 0; jj < NB / 2; ++jj) {
          const float other = xchg[jj * 128 + mate], mine = gate ? v[jj] : v[NB / 2 + jj];
          const float g = gate ? mine : other, u = gate ? other : mine;
          ty[(j0 + jj) * 68 + (row & 63)] = __fdividef(g, 1.0f + __expf(-g)) * u;
        }
        epi_sync();
        if (lane < a.batch) {
          float y[16];
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const float4 t = *reinterpret_cast<const float4*>(ty + lane * 68 + q * 16 + 4 * c);
            y[4 * c] = t.x;
            y[4 * c + 1] = t.y;
            y[4 * c + 2] = t.z;
            y[4 * c + 3] = t.w;
          }
          const size_t off = lane * width + (size_t)tile * 64 + q * 16;
          if (a.dtype == DOE_DTYPE_F32) {
            float4* o = reinterpret_cast<float4*>(static_cast<float*>(a.out[0]) + off);
#pragma unroll
            for (int c = 0; c < 4; ++c) o[c] = make_float4(y[4 * c], y[4 * c + 1], y[4 * c + 2], y[4 * c + 3]);
          } else {
            uint4* o = reinterpret_cast<uint4*>(static_cast<uint16_t*>(a.out[0]) + off);
            o[0] = pack8(y, a.dtype == DOE_DTYPE_BF16);
            o[1] = pack8(y + 8, a.dtype == DOE_DTYPE_BF16);
          }
        }
        // the next writes to ty come after the next segment's first barrier
        // the next writes to xchg come after the next segment's epi_all
      } else {
        const int col0 = (int)tile * BM;
        const int sg = col0 < a.seg_end[0] ? 0 : (col0 < a.seg_end[1] ? 1 : 2);
        const int base = sg == 0 ? 0 : (sg == 1 ? a.seg_end[0] : a.seg_end[1]);
        const size_t width = (size_t)((sg == 0 ? a.seg_end[0] : (sg == 1 ? a.seg_end[1] : a.seg_end[2])) - base);
        void* dst = sg == 0 ? a.out[0] : (sg == 1 ? a.out[1] : a.out[2]);
        if (a.residual) {
          // each residual element is loaded by the thread of its column before
          // the transpose below, and stored after it: an in-place residual
          // (out[0] == residual) stays correct
          if (!pre_res) {
            const int col = col0 + row;
#pragma unroll
            for (int j = 0; j < NB; ++j) rres[j] = j < a.batch ? a.residual[(size_t)j * a.n_out + col] : 0.0f;
          }
#pragma unroll
          for (int j = 0; j < NB; ++j) v[j] += rres[j];
        }
        // Transpose the warp's 32 columns x 32 batch rows through its own 32
        // lines of the receive area (unused outside cluster mode; in cluster
        // mode this warp's lines of slot 0, already added up), so that lane j
        // holds batch row j's 32 consecutive columns and writes them with
        // 16-byte stores: a few dozen instructions on the launch's tail
        // instead of 32 scalar stores per thread.  Column c of row j sits in
        // 16-byte chunk (c / 4) ^ (j % 8) of line j (no bank conflicts).
        float* tl = reinterpret_cast<float*>(smem + OFF_RECV + (uint32_t)q * 32 * 128);
        __syncwarp();
#pragma unroll
        for (int j = 0; j < NB; ++j) tl[j * 32 + ((((lane >> 2) ^ (j & 7)) << 2) | (lane & 3))] = v[j];
        __syncwarp();
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const float4 t = *reinterpret_cast<const float4*>(tl + lane * 32 + ((c ^ (lane & 7)) << 2));
          v[4 * c] = t.x;
          v[4 * c + 1] = t.y;
          v[4 * c + 2] = t.z;
          v[4 * c + 3] = t.w;
        }
        if (a.normed_out != nullptr) asm volatile("cp.async.wait_all;\n" ::: "memory");
        __syncwarp();  // the lines are free again for the next segment; gamma has landed
        const int cw = col0 + q * 32;  // the warp's first column
        if (lane < a.batch) {
          if (a.dtype == DOE_DTYPE_F32) {
            float4* o = reinterpret_cast<float4*>(static_cast<float*>(dst) + lane * width + (cw - base));
#pragma unroll
            for (int c = 0; c < 8; ++c) o[c] = make_float4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
          } else {
            uint4* o = reinterpret_cast<uint4*>(static_cast<uint16_t*>(dst) + lane * width + (cw - base));
#pragma unroll
            for (int c = 0; c < 4; ++c) o[c] = pack8(v + 8 * c, a.dtype == DOE_DTYPE_BF16);
          }
          if (a.normed_out != nullptr) {
            // producer of a split RMSNorm (f32, one segment): bf16(y * gamma)
            // and row `lane`'s sum of y^2 over the warp's 32 columns, in order
            uint4* o = reinterpret_cast<uint4*>(a.normed_out + (size_t)lane * a.n_out + cw);
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              const uint4 g4 = *reinterpret_cast<const uint4*>(smem + OFF_XCHG + q * 64 + c * 16);
              const uint32_t gw[4] = {g4.x, g4.y, g4.z, g4.w};
              float y[8];
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float2 g2 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&gw[e]));
                y[2 * e] = v[8 * c + 2 * e] * g2.x;
                y[2 * e + 1] = v[8 * c + 2 * e + 1] * g2.y;
              }
              o[c] = pack8(y, true);
            }
            float ss = 0.0f;
#pragma unroll
            for (int i = 0; i < 32; ++i) ss += v[i] * v[i];
            a.ssq_out[(size_t)(cw >> 5) * NB + lane] = ss;
          }
        } else if (a.normed_out != nullptr) {
          a.ssq_out[(size_t)(cw >> 5) * NB + lane] = 0.0f;  // rows past batch
        }
      }
    }
  }

  // no copy of gamma may land after the CTA exits
  if (warp >= 2 && a.normed_out != nullptr) asm volatile("cp.async.wait_all;\n" ::: "memory");
  // cluster rank 0 keeps its shared memory until every remote store has
  // landed, also when it stopped early (bounded)
  if (a.cluster > 1 && warp >= 2 && recv_bytes((int)crank, a) > 0) mbar_wait_bounded(bar(RECV_FULL), 0);
  tc_fence_before();
  __syncthreads();
  // no CTA of a cluster leaves before rank 0 holds every accumulator
  if (a.cluster > 1) cluster_sync_all();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem), "r"(kTmemCols));
  }
}

// out[r, :] = bf16(x[r, :] * (1 / sqrt(mean(x[r, :]^2) + eps)) * gamma)
constexpr int kNormThreads = 256;
__global__ void __launch_bounds__(kNormThreads) rmsnorm_kernel(const float* __restrict__ x,
                                                               const __nv_bfloat16* __restrict__ gamma,
                                                               __nv_bfloat16* __restrict__ out, int cols,
                                                               float eps) {
  __shared__ float warp_sum[kNormThreads / 32];
  pdl_trigger();
  pdl_wait();
  const size_t row = blockIdx.x;
  const float4* xr = reinterpret_cast<const float4*>(x + row * cols);
  const int n4 = cols >> 2;
  float ss = 0.0f;
  for (int i = threadIdx.x; i < n4; i += kNormThreads) {
    const float4 v = xr[i];
    ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) warp_sum[threadIdx.x >> 5] = ss;
  __syncthreads();
  float total = 0.0f;
#pragma unroll
  for (int w = 0; w < kNormThreads / 32; ++w) total += warp_sum[w];
  const float inv = 1.0f / sqrtf(total / (float)cols + eps);
  const uint2* g2 = reinterpret_cast<const uint2*>(gamma);
  uint2* o2 = reinterpret_cast<uint2*>(out + row * cols);
  for (int i = threadIdx.x; i < n4; i += kNormThreads) {
    const float4 v = xr[i];
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

}  // namespace lin

// ---- host -----------------------------------------------------------------
int current_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    cudaGetLastError();
    set_op_error("no current CUDA device (or its ordinal is %d or more)", kMaxDevices);
    return -1;
  }
  return dev;
}

// SM count of the current device (cached per device).
int num_sms() {
  static std::atomic<int> cached[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    cudaGetLastError();
    return 148;
  }
  if (cached[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      n = 148;
    }
    cached[dev].store(n);
  }
  return cached[dev].load();
}

namespace {


// Workspace layout, the same for every shape so that calls of different
// sizes can share one workspace: tile counters at the front (room for
// kMaxTiles tiles), partial tiles from kCountersBytes on.
constexpr uint64_t kMaxTiles = 16384;
constexpr uint64_t kCountersBytes = kMaxTiles * 4;

// Clusters of `size` linear CTAs that fit on the device at once (cached per
// device and size); -1 with the op error set on failure.
// The kernel's dynamic shared-memory limit, raised once per device.
int set_smem_attr(int dev) {
  static std::atomic<bool> done[64];
  if (done[dev].load()) return DOE_OK;
  int rc = cuda_status(cudaFuncSetAttribute(lin::linear_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            lin::kSmemBytes),
                       "cudaFuncSetAttribute(linear)");
  if (rc == DOE_OK) done[dev].store(true);
  return rc;
}

int max_active_clusters(int size) {
  static std::atomic<int> cached[64][lin::kMaxCluster + 1];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    cudaGetLastError();
    set_op_error("doe_linear_bf16: no current device");
    return -1;
  }
  const int have = cached[dev][size].load();
  if (have != 0) return have < 0 ? 0 : have;
  if (set_smem_attr(dev) != DOE_OK) return -1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)size);
  cfg.blockDim = dim3(lin::kThreads);
  cfg.dynamicSmemBytes = lin::kSmemBytes;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)size;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cuda_status(cudaOccupancyMaxActiveClusters(&n, lin::linear_kernel, &cfg), "cudaOccupancyMaxActiveClusters") !=
      DOE_OK)
    return -1;
  cached[dev][size].store(n > 0 ? n : -2);  // -2: none fit (never chosen)
  return n > 0 ? n : 0;
}

}  // namespace

uint64_t linear_workspace(uint32_t n_out, uint32_t k) {
  (void)n_out;
  (void)k;
  return kCountersBytes + (uint64_t)lin::kMaxCtas * 2 * lin::NB * lin::BM * sizeof(float);
}

int launch_linear(const void* x, const void* w, uint32_t batch, uint32_t n_out, uint32_t k,
                  const doe_linear_out* o, const doe_linear_norm* norm, const doe_launch* launch) {
  const uint32_t tiles = n_out / lin::BM, kb = k / lin::BK;
  if (tiles > kMaxTiles) {
    set_op_error("doe_linear_bf16: n_out %u exceeds %llu rows", n_out, (unsigned long long)(kMaxTiles * lin::BM));
    return DOE_UNSUPPORTED;
  }
  if (k % lin::BK != 0) {
    set_op_error("doe_linear_bf16: k %u must be a multiple of %d", k, lin::BK);
    return DOE_UNSUPPORTED;
  }
  const long long iters = (long long)tiles * kb;
  const int sms = num_sms();
  // Fewer tiles than half the SMs: split each tile's k over a cluster of up to
  // kMaxCluster CTAs that sum through distributed shared memory.  Otherwise
  // stream-K over the whole product.
  // The tile's clusters must all be resident at once (one CTA per SM, a
  // cluster's CTAs on one GPC), or the split costs a second wave.
  int cluster = 1;
  if ((long long)tiles * 2 <= sms) {
    int c = sms / (int)tiles;
    if (c > lin::kMaxCluster) c = lin::kMaxCluster;
    if (c > (int)(kb / lin::kMinIters)) c = (int)(kb / lin::kMinIters);
    for (; c > 1; --c) {
      const int fit = max_active_clusters(c);
      if (fit < 0) return DOE_CUDA_ERROR;
      if ((int)tiles <= fit) break;
    }
    cluster = c;
  }
  int ctas;
  if (cluster > 1) {
    ctas = (int)tiles * cluster;
  } else {
    cluster = 1;
    ctas = sms * lin::kCtasPerSm;
    if (ctas > lin::kMaxCtas) ctas = lin::kMaxCtas;
    // enough stages per CTA to cover the load latency, few CTAs per tile so the
    // partial-tile reduction stays short
    long long cap = iters / lin::kMinIters > 0 ? iters / lin::kMinIters : 1;
    if (cap > (long long)tiles * lin::kMaxSplit) cap = (long long)tiles * lin::kMaxSplit;
    if ((long long)ctas > cap) ctas = (int)cap;
  }
  const uint64_t need = linear_workspace(n_out, k);
  if (launch->workspace == nullptr || launch->workspace_bytes < need) {
    set_op_error("doe_linear_bf16: workspace of %llu bytes required, %llu given", (unsigned long long)need,
                 (unsigned long long)launch->workspace_bytes);
    return DOE_INVALID_ARGUMENT;
  }
  lin::Args a;
  int end = 0;
  for (int i = 0; i < 3; ++i) {
    a.out[i] = o->out[i];
    end += (int)o->width[i];
    a.seg_end[i] = o->width[i] ? end : 0x7fffffff;
  }
  a.residual = o->residual;
  a.counters = static_cast<unsigned*>(launch->workspace);
  a.part = reinterpret_cast<float*>(static_cast<uint8_t*>(launch->workspace) + kCountersBytes);
  a.status = launch->status;
  a.batch = (int)batch;
  a.n_out = (int)n_out;
  a.kb = (int)kb;
  a.tiles = (int)tiles;
  a.ctas = ctas;
  a.epilogue = (int)o->epilogue;
  a.dtype = (int)o->dtype;
  a.iters = iters;
  a.cluster = cluster;
  a.gamma_out = norm ? static_cast<const __nv_bfloat16*>(norm->gamma) : nullptr;
  a.normed_out = norm && norm->gamma ? static_cast<__nv_bfloat16*>(norm->normed_out) : nullptr;
  a.ssq_out = norm && norm->gamma ? norm->ssq_out : nullptr;
  a.ssq_in = norm ? norm->ssq_in : nullptr;
  a.eps = norm ? norm->eps : 0.0f;
  CUtensorMap mw, mx;
  int rc = encode_rows_map(&mw, w, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, k, 1, n_out, 64, lin::BM,
                           "doe_linear_bf16");
  if (rc == DOE_OK)
    rc = encode_rows_map(&mx, x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, k, 1, batch, 64, lin::NB,
                         "doe_linear_bf16");
  if (rc != DOE_OK) return rc;
  {
    int dev = 0;
    rc = cuda_status(cudaGetDevice(&dev), "cudaGetDevice");
    if (rc == DOE_OK && (dev < 0 || dev >= 64)) {
      set_op_error("doe_linear_bf16: device ordinal %d beyond 63", dev);
      rc = DOE_UNSUPPORTED;
    }
    if (rc == DOE_OK) rc = set_smem_attr(dev);
    if (rc != DOE_OK) return rc;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(ctas);
  cfg.blockDim = dim3(lin::kThreads);
  cfg.dynamicSmemBytes = lin::kSmemBytes;
  cfg.stream = static_cast<cudaStream_t>(launch->stream);
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = (unsigned)cluster;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cuda_status(cudaLaunchKernelEx(&cfg, lin::linear_kernel, mw, mx, a), "linear_kernel");
}

int launch_rmsnorm(const float* x, const void* gamma, float eps, void* out, uint32_t rows, uint32_t cols,
                   const doe_launch* launch) {
  return cuda_status(launch_pdl(lin::rmsnorm_kernel, dim3(rows), dim3(lin::kNormThreads), 0,
                                static_cast<cudaStream_t>(launch->stream), x,
                                static_cast<const __nv_bfloat16*>(gamma), static_cast<__nv_bfloat16*>(out),
                                (int)cols, eps),
                     "rmsnorm_kernel");
}

}  // namespace doe
