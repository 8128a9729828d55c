// prefill_sm100.cu -- causal prefill attention on the 5th-generation tensor
// cores (tcgen05 + TMEM + TMA), with the prompt's K/V written into a paged
// KV cache on the way.
//
// Semantics: attention_head256_f16kv.wgsl with query_len = seq_len,
// is_causal, start_pos = kv_start = 0, dense K/V (…wgsl:113-136 key bounds,
// 181-217 online softmax, 257-268 out = acc / l), f16 Q/K/V in [S, H, D]
// ([B,S,H,D] with B = 1), f32 accumulation and f32 output; GQA kv head =
// h / (H / Hkv).  The cache write is kv_write generalised to the paged pool
// (runtime/zig/src/tsir/emit_kernel_body.zig:620-690).
//
// Persistent: one CTA per SM walks a list of work items, each a pair of
// 128-row query tiles (A = 2m, B = 2m+1) of one head; the items are numbered
// heaviest first and dealt out zig-zag (CTA c takes item rG + c in even rounds
// and rG + G - 1 - c in odd ones), so heavy and light items pair up.  The two
// tiles of an item share every K/V tile.  512 threads in four warpgroups:
//   warps 0-3   softmax of tile A, warps 4-7 softmax of tile B: one thread
//               per query row (TMEM lane), holding all 128 scores of a key
//               tile in registers (setmaxnreg: 176 registers each, taken
//               from the epilogue and control warpgroups).  Once a row has a
//               running max, keys [0, 64) are exponentiated against it while
//               the tile's max is reduced; P (f16) goes over the S columns it
//               came from, keys [0, 64) published on P_HALF_x as soon as they
//               land, keys [64, 128) on P_FULL_x.  The running max moves only
//               when a row's max rises by more than 2^8 (O is then rescaled
//               in TMEM and that tile's first half recomputed).
//   warps 8-11  epilogue: O_x / l -> f32 rows, staged 32 x 32 in shared
//               memory and TMA-stored, while the next item already runs;
//               then O_x is handed back (O_EMPTY_x)
//   warp 12     TMEM owner + MMA issuer (whole warp, one elected lane issues):
//               S_A = Q_A K^T, S_B = Q_B K^T, then O_A += P_A V and O_B +=
//               P_B V, ping-ponging so the tensor core works on one tile while
//               the other tile's softmax runs; each PV runs in two halves
//   warp 13     TMA producer: Q_A, Q_B per item, K and V tiles into two 2-slot
//               rings that run on across items (K a tile ahead of V); it also
//               TMA-stores the diagonal K/V tiles into the paged cache
//   warps 14-15 no work (their registers go to the softmax warpgroups)
// TMEM: S_A [0,128) S_B [128,256) O_A [256,384) O_B [384,512); P_x aliases
// the first 64 columns of S_x.  A commit on S_x(j+1) covers PV_x(j), so when
// a softmax warp sees S_x(j+1) its P buffer is free and O_x is quiescent.
// Operands: Q, K K-major SWIZZLE_128B smem tiles; V an MN-major smem tile;
// P from TMEM.  No cluster multicast.  Every mbarrier wait is bounded (~2 s
// of clock cycles); on timeout the kernel records DOE_DEVICE_ERR_TIMEOUT, the
// roles stop, all issued MMAs are waited for (bounded) and TMEM is freed.
// There is no named barrier: a role that stops early only skips mbarrier
// arrivals, which the others' bounded waits absorb.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "tma.cuh"
#include "umma.cuh"

namespace doe {
namespace pf {

constexpr int BM = 128, BN = 128, HD = 128;
constexpr int kThreads = 512;  // softmax A, softmax B, epilogue, MMA + TMA (+ 2 idle) warpgroups
constexpr int kEpiWarp0 = 8, kMmaWarp = 12, kTmaWarp = 13;
// setmaxnreg split of the 512 x 128 launch registers: softmax warpgroups
// 2 x 128 x 176, epilogue 128 x 64, MMA / TMA warpgroup 128 x 96 = 65,536 (no spills)
constexpr int kSoftmaxRegs = 176, kEpiRegs = 64, kCtlRegs = 96;
constexpr uint32_t kSub = 128 * 128;      // one 128-row x 64-half swizzled sub-tile (16 KB)
constexpr uint32_t kTile = 2 * kSub;      // 128 x 128 f16 tile (32 KB)
constexpr uint32_t OFF_Q = 0;                        // Q_A, Q_B
constexpr uint32_t OFF_K = OFF_Q + 2 * kTile;        // 2 stages
constexpr uint32_t OFF_V = OFF_K + 2 * kTile;        // 2 stages
constexpr uint32_t OFF_BAR = OFF_V + 2 * kTile;      // barriers + TMEM slot
constexpr uint32_t OFF_L = OFF_BAR + 256;            // row sums handed to the epilogue: [tile][item & 1][128]
constexpr uint32_t OFF_EPI = (OFF_L + 2 * 2 * 128 * 4 + 1023) & ~1023u;  // 4 x 4 KB output staging
constexpr uint32_t kEpiStage = 32 * 32 * 4;          // 32 rows x 32 f32 columns, 128-byte swizzle
constexpr uint32_t kSmemBytes = OFF_EPI + 4 * kEpiStage + 1024;  // + alignment slack
constexpr uint32_t kTmemCols = 512;
constexpr long long kWaitCycles = 4000000000LL;      // ~2 s at 1.9 GHz
constexpr uint32_t kSuspendNs = 20000;                // try_wait sleep hint (the 2 s bound is checked between)

// Barriers live for the whole kernel: each role counts the phases of the
// ones it waits on across work items.
enum Bar { Q_FULL, Q_EMPTY, K_FULL0, K_FULL1, V_FULL0, V_FULL1, K_EMPTY0, K_EMPTY1, V_EMPTY0, V_EMPTY1,
           S_FULL_A, S_FULL_B, P_HALF_A, P_HALF_B, P_FULL_A, P_FULL_B, O_FULL_A, O_FULL_B,
           O_EMPTY_A, O_EMPTY_B, L_READY_A, L_READY_B, MMA_DONE, NUM_BARS };

struct Args {
  float* out;               // [S, H, D] f32
  int32_t* status;
  const int32_t* table;     // block-table row of the cache sequence (or null)
  int seq_len, num_heads, num_kv_heads, n_qtiles, n_pairs, causal;
  int num_items;            // n_pairs * num_heads (query-tile pair, head) items, heaviest first
  int cache_page_size, cache_num_pages, cache_max_pages, cache_start;
  float scale_log2;
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(bar), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(bar), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n.reg .pred p;\n"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      "selp.b32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// try_wait with a suspend-time hint: a thread whose phase is not complete
// sleeps in hardware until it completes (or kSuspendNs pass) instead of
// re-polling; polling warps take shared-memory bandwidth from the SS MMAs.
__device__ __forceinline__ bool mbar_try_sleep(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n.reg .pred p;\n"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
      "selp.b32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "r"(kSuspendNs)
      : "memory");
  return ok != 0;
}
// Bounded wait: false (and an error bit, and the CTA abort flag) on timeout.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                          int32_t* status) {
  if (mbar_try(bar, parity)) return true;
  const long long t0 = clock64();
  while (true) {
    if (mbar_try_sleep(bar, parity)) return true;
    if (*abort_flag) return false;
    if (clock64() - t0 > kWaitCycles) {
      *abort_flag = 1;
      report(status, DOE_DEVICE_ERR_TIMEOUT);
      return false;
    }
  }
}

// max(a, b, c) in one instruction (sm_100), NaN handling as fmaxf.
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;\n" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// 2^x with the SFU's approximate exp2 (max relative error ~2^-22); -inf -> +0.
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;\n" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                            int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];\n" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, uint32_t src, int x, int y,
                                             int z) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];\n" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(src), "r"(x), "r"(y), "r"(z)
               : "memory");
}

// The (query-tile pair, head) work item `it`: items are numbered heaviest
// first (the pair with the longest key range first, heads inside a pair).
struct Item {
  int h, hk, tA, tB, nA, nB, n_kv;
  bool hasB;
};
__device__ __forceinline__ Item item_of(const Args& a, int it) {
  Item t;
  const int H = a.num_heads;
  const int order = it / H;
  t.h = it - order * H;
  const int pair = a.n_pairs - 1 - order;
  t.hk = t.h / (H / a.num_kv_heads);
  const int n_kv_all = (a.seq_len + BN - 1) / BN;
  t.tA = 2 * pair;
  t.tB = 2 * pair + 1;
  t.hasB = t.tB < a.n_qtiles;
  t.nA = a.causal ? t.tA + 1 : n_kv_all;
  t.nB = t.hasB ? (a.causal ? t.tB + 1 : n_kv_all) : 0;
  t.n_kv = t.nA > t.nB ? t.nA : t.nB;
  return t;
}
// The r-th item of CTA c in a grid of G: items rG + c in even rounds and
// rG + G - 1 - c in odd ones (a zig-zag over the heaviest-first order, so a
// CTA that takes a heavy item in one round takes a light one in the next);
// -1 past the last item.
__device__ __forceinline__ int nth_item(const Args& a, int r) {
  const int G = (int)gridDim.x, c = (int)blockIdx.x;
  const int it = r * G + ((r & 1) ? G - 1 - c : c);
  return it < a.num_items ? it : -1;
}

__global__ void __launch_bounds__(kThreads, 1)
    prefill_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                   const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_ck,
                   const __grid_constant__ CUtensorMap tm_cv, const __grid_constant__ CUtensorMap tm_o,
                   const Args a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + OFF_BAR + 8 * NUM_BARS);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + OFF_BAR + 8 * NUM_BARS + 8);
  float* l_sm = reinterpret_cast<float*>(smem + OFF_L);
  auto bar = [&](int i) { return smem_u32(&bars[i]); };

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int H = a.num_heads;

  if (threadIdx.x == 0) {
    // P_HALF_x / P_FULL_x / L_READY_x: one arrival from each of tile x's 4
    // softmax warps; O_EMPTY_x: one from each of the 4 epilogue warps
    for (int i = 0; i < NUM_BARS; ++i)
      mbar_init(bar(i), ((i >= P_HALF_A && i <= P_FULL_B) || (i >= O_EMPTY_A && i <= L_READY_B)) ? 4u : 1u);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  if (warp == kMmaWarp) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // registers: the softmax warpgroups take what the other two give up; each
  // role's code sits inside the branch that sets its register count
  if (warp >= kMmaWarp) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;\n" ::"n"(kCtlRegs));
    if (warp == kTmaWarp && lane == 0) {
      // ---------------------------------------------------------- producer
      // K runs one tile ahead of V: the MMA issuer is done with K(j) an
      // iteration before it is done with V(j), so each ring slot is refilled
      // as soon as its own tile is released.  The rings run on across items:
      // g counts the tiles of a ring loaded so far, slot g & 1, and tile g is
      // released by the (g/2)-th arrival on its slot's EMPTY barrier.
      uint32_t gk = 0, gv = 0;
      bool ok = true;
      auto load = [&](int ring, uint32_t g, int hk, int row) -> bool {
        const int st = g & 1;
        if (g >= 2 &&
            !mbar_wait(bar((ring == 0 ? K_EMPTY0 : V_EMPTY0) + st), ((g >> 1) - 1) & 1, abort_flag, a.status))
          return false;
        const uint32_t full = bar((ring == 0 ? K_FULL0 : V_FULL0) + st);
        const uint32_t dst = sbase + (ring == 0 ? OFF_K : OFF_V) + st * kTile;
        const CUtensorMap* map = ring == 0 ? &tm_k : &tm_v;
        mbar_expect_tx(full, kTile);
        tma_load_3d(dst, map, full, 0, hk, row);
        tma_load_3d(dst + kSub, map, full, 64, hk, row);
        return true;
      };
      for (int r = 0; ok; ++r) {
        const int it = nth_item(a, r);
        if (it < 0) break;
        const Item t = item_of(a, it);
        // Q of the previous item is free once its last S MMAs are done
        if (r > 0 && !(ok = mbar_wait(bar(Q_EMPTY), (r - 1) & 1, abort_flag, a.status))) break;
        mbar_expect_tx(bar(Q_FULL), (t.hasB ? 2 : 1) * kTile);
        tma_load_3d(sbase + OFF_Q, &tm_q, bar(Q_FULL), 0, t.h, t.tA * BM);
        tma_load_3d(sbase + OFF_Q + kSub, &tm_q, bar(Q_FULL), 64, t.h, t.tA * BM);
        if (t.hasB) {
          tma_load_3d(sbase + OFF_Q + kTile, &tm_q, bar(Q_FULL), 0, t.h, t.tB * BM);
          tma_load_3d(sbase + OFF_Q + kTile + kSub, &tm_q, bar(Q_FULL), 64, t.h, t.tB * BM);
        }
        const uint32_t k0 = gk, v0 = gv;
        ok = load(0, gk++, t.hk, 0);
        for (int j = 0; j < t.n_kv && ok; ++j) {
          if (j + 1 < t.n_kv) ok = load(0, gk++, t.hk, (j + 1) * BN);
          if (ok) ok = load(1, gv++, t.hk, j * BN);
        }
        // causal: the key tiles tA and tB are this item's diagonals; the first
        // head of each kv group writes their K/V rows into the paged cache
        // (16-row boxes: one page slice each).  Both are the last two tiles
        // loaded, so they still sit in the rings.
        if (ok && a.table != nullptr && a.causal && (t.h % (H / a.num_kv_heads)) == 0) {
          for (int j = (t.n_kv >= 2 ? t.n_kv - 2 : 0); j < t.n_kv && ok; ++j) {
            if (j != t.tA && j != t.tB) continue;
            const uint32_t gkj = k0 + j, gvj = v0 + j;
            ok = mbar_wait(bar(K_FULL0 + (gkj & 1)), (gkj >> 1) & 1, abort_flag, a.status) &&
                 mbar_wait(bar(V_FULL0 + (gvj & 1)), (gvj >> 1) & 1, abort_flag, a.status);
            if (!ok) break;
            asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
            for (int m = 0; m < BN / 16; ++m) {
              const int tok = j * BN + m * 16;
              if (tok + 16 > a.seq_len) break;
              const int pos = a.cache_start + tok;
              const int pidx = pos / a.cache_page_size;
              const int page = pidx < a.cache_max_pages ? a.table[pidx] : -1;
              if ((unsigned)page >= (unsigned)a.cache_num_pages) {
                report(a.status, DOE_DEVICE_ERR_PAGE);
                continue;
              }
              const int row = page * a.cache_page_size + (pos - pidx * a.cache_page_size);
              for (int sub = 0; sub < 2; ++sub) {
                const uint32_t m_off = sub * kSub + m * 16 * 128;
                tma_store_3d(&tm_ck, sbase + OFF_K + (gkj & 1) * kTile + m_off, sub * 64, t.hk, row);
                tma_store_3d(&tm_cv, sbase + OFF_V + (gvj & 1) * kTile + m_off, sub * 64, t.hk, row);
              }
            }
          }
          // the stores have read their ring slots before the next loads refill them
          asm volatile("cp.async.bulk.commit_group;\n" ::: "memory");
          asm volatile("cp.async.bulk.wait_group.read 0;\n" ::: "memory");
        }
      }
      asm volatile("cp.async.bulk.wait_group 0;\n" ::: "memory");
    } else if (warp == kMmaWarp) {
      // ---------------------------------------------------------- MMA issuer
      // The whole warp runs the (warp-uniform) control flow and one elected
      // lane issues each tcgen05 instruction: the descriptors stay in uniform
      // registers and each MMA costs an add and the issue itself.
      const uint32_t idq = idesc_f16(false), idp = idesc_f16(true);
      const uint64_t dq = sdesc(sbase + OFF_Q, 16, 1024);      // Q_A; Q_B is kTile further
      const uint64_t dk = sdesc(sbase + OFF_K, 16, 1024);      // K ring slot 0
      const uint64_t dv = sdesc(sbase + OFF_V, kSub, 1024);    // V ring slot 0
      // S_x = Q_x K^T (K tile in ring slot st) into TMEM columns [128x, 128x + 128)
      auto issue_s = [&](int x, int st) {
        const uint64_t q = dq + ((x * kTile) >> 4), k = dk + ((st * kTile) >> 4);
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint32_t off = ((kk >> 2) * kSub + (kk & 3) * 32) >> 4;  // start-address field units
          umma_elect(tmem + x * 128, q + off, k + off, idq, kk > 0);
        }
        commit_elect(bar(S_FULL_A + x));
      };
      // O_x (+)= P_x V with P_x (f16) in TMEM columns [128x, 128x + 64), keys
      // 2c and 2c + 1 in column c: part 0 is keys [0, 64) (published on
      // P_HALF_x), part 1 keys [64, 128); `first`: the item's first PV_x,
      // which overwrites O_x
      auto issue_pv = [&](int x, int st, int part, bool first) {
        const uint64_t v = dv + ((st * kTile) >> 4);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int kk = part * 4 + i;  // 16-key slice
          umma_ts_elect(tmem + 256 + x * 128, tmem + x * 128 + kk * 8, v + ((kk * 16 * 128) >> 4), idp,
                        (!first || part > 0 || i > 0) ? 1u : 0u);
        }
      };
      // bounded wait by every lane, agreed across the warp so it stays converged
      auto wait = [&](int b, uint32_t parity) {
        return __all_sync(0xffffffffu, mbar_wait(bar(b), parity, abort_flag, a.status));
      };
      uint32_t gk = 0, gv = 0;          // K / V tiles consumed so far
      uint32_t ph[2] = {0, 0};          // P phases per tile (S_FULL / P_HALF / P_FULL steps)
      uint32_t nitems[2] = {0, 0};      // items done per tile (O_FULL / O_EMPTY phases)
      bool ok = true;
      for (int r = 0; ok; ++r) {
        const int it = nth_item(a, r);
        if (it < 0) break;
        const Item t = item_of(a, it);
        const int nt[2] = {t.nA, t.nB};
        ok = wait(Q_FULL, r & 1) && wait(K_FULL0 + (gk & 1), (gk >> 1) & 1);
        if (!ok) break;
        tc_fence_after();
        // S_x(0) may run at once: the previous item's P_x has been consumed
        // (its PV_x was issued before this) and its softmax has read S_x
        issue_s(0, gk & 1);
        if (t.nB > 0) issue_s(1, gk & 1);
        commit_elect(bar(K_EMPTY0 + (gk & 1)));  // K released once S_x(0) are done
        if (t.n_kv == 1) commit_elect(bar(Q_EMPTY));
        for (int j = 0; j < t.n_kv && ok; ++j) {
          const uint32_t kj = gk + j, vj = gv + j;
          ok = wait(V_FULL0 + (vj & 1), (vj >> 1) & 1);
          bool k_ready = false;  // K(j+1) seen complete
          for (int x = 0; x < 2 && ok; ++x) {
            if (j >= nt[x]) continue;
            // every mbarrier wait here costs the issue stream ~100 cycles even
            // when the phase is complete, so each is taken only once per step
            ok = wait(P_HALF_A + x, ph[x] & 1);
            if (ok && j == 0 && nitems[x] > 0) ok = wait(O_EMPTY_A + x, (nitems[x] - 1) & 1);
            if (!ok) break;
            tc_fence_after();
            issue_pv(x, vj & 1, 0, j == 0);
            ok = wait(P_FULL_A + x, ph[x] & 1);
            if (!ok) break;
            ++ph[x];
            tc_fence_after();
            issue_pv(x, vj & 1, 1, j == 0);
            if (j == nt[x] - 1) {
              commit_elect(bar(O_FULL_A + x));
              ++nitems[x];
            } else {
              if (!k_ready) {
                ok = wait(K_FULL0 + ((kj + 1) & 1), ((kj + 1) >> 1) & 1);
                if (!ok) break;
                k_ready = true;
              }
              tc_fence_after();
              issue_s(x, (kj + 1) & 1);
            }
          }
          if (!ok) break;
          if (j + 1 < t.n_kv) commit_elect(bar(K_EMPTY0 + ((kj + 1) & 1)));  // K(j+1): S_x(j+1) issued
          if (j + 2 == t.n_kv) commit_elect(bar(Q_EMPTY));                    // the item's last S issued
          commit_elect(bar(V_EMPTY0 + (vj & 1)));                             // V(j): PV_x(j) issued
        }
        gk += t.n_kv;
        gv += t.n_kv;
      }
      // every MMA this warp issued has finished once MMA_DONE flips
      commit_elect(bar(MMA_DONE));
      wait(MMA_DONE, 0);
    }
  } else if (warp >= kEpiWarp0) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;\n" ::"n"(kEpiRegs));
    // ------------------------------------------------------------ epilogue
    // O_x / l -> f32 rows, item by item, while the softmax warps and the
    // tensor core already work on the next item; then O_x is handed back.
    // Each warp stages its 32 rows, 32 columns at a time, in its own 4 KB
    // buffer (128-byte swizzle: 16-byte chunk k of row r at chunk k ^ (r & 7),
    // so the 32 lanes' row writes spread over all banks) and one lane
    // TMA-stores the box; rows past seq_len are clipped by the tensor map.
    // Whole-line writes keep the L1/shared-memory path free for the tensor
    // core's operand reads, which row-per-lane global stores would contend with.
    const int wl = warp & 3;
    const int row = wl * 32 + lane;
    const uint32_t lane_base = tmem + ((uint32_t)(wl * 32) << 16);
    uint8_t* stage_p = smem + OFF_EPI + wl * kEpiStage;
    const uint32_t stage = sbase + OFF_EPI + wl * kEpiStage;
    uint32_t nitems[2] = {0, 0};
    bool ok = true;
    for (int r = 0; ok; ++r) {
      const int it = nth_item(a, r);
      if (it < 0) break;
      const Item t = item_of(a, it);
      for (int x = 0; x < 2 && ok; ++x) {
        if ((x == 0 ? t.nA : t.nB) == 0) continue;
        const uint32_t n = nitems[x]++;
        ok = __all_sync(0xffffffffu, mbar_wait(bar(O_FULL_A + x), n & 1, abort_flag, a.status) &&
                                         mbar_wait(bar(L_READY_A + x), n & 1, abort_flag, a.status));
        if (!ok) break;
        tc_fence_after();
        const float l = l_sm[(x * 2 + (n & 1)) * 128 + row];
        const float inv = l > 0.0f ? 1.0f / l : 0.0f;
        const int row0 = (x == 0 ? t.tA : t.tB) * BM + wl * 32;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t o[32];
          tmem_ld32(lane_base + 256 + x * 128 + c * 32, o);
          tmem_wait_ld();
          // the previous box's store has finished reading the buffer
          if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 0;\n" ::: "memory");
          __syncwarp();
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const float4 v = make_float4(__uint_as_float(o[4 * k]) * inv, __uint_as_float(o[4 * k + 1]) * inv,
                                         __uint_as_float(o[4 * k + 2]) * inv, __uint_as_float(o[4 * k + 3]) * inv);
            *reinterpret_cast<float4*>(stage_p + lane * 128 + ((k ^ (lane & 7)) << 4)) = v;
          }
          asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
          __syncwarp();
          if (lane == 0) {
            tma_store_3d(&tm_o, stage, c * 32, t.h, row0);
            asm volatile("cp.async.bulk.commit_group;\n" ::: "memory");
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(O_EMPTY_A + x));
      }
    }
    if (lane == 0) asm volatile("cp.async.bulk.wait_group 0;\n" ::: "memory");
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;\n" ::"n"(kSoftmaxRegs));
    // ------------------------------------------------------------ softmax
    const int x = warp >> 2;                 // tile A (x = 0) or B (x = 1)
    const int wl = warp & 3;                 // TMEM lane group
    const int row = wl * 32 + lane;
    const uint32_t lane_base = tmem + ((uint32_t)(wl * 32) << 16);
    const uint32_t s_col = x * 128, o_col = 256 + x * 128;
    uint32_t ph = 0, nitems = 0;
    bool ok = true;
    for (int r = 0; ok; ++r) {
      const int it = nth_item(a, r);
      if (it < 0) break;
      const Item t = item_of(a, it);
      const int nt = x == 0 ? t.nA : t.nB;
      if (nt == 0) continue;
      const int q_idx = (x == 0 ? t.tA : t.tB) * BM + row;
      float m_used = -INFINITY, l = 0.0f;
      for (int j = 0; j < nt && ok; ++j, ++ph) {
        // S_x(j) is ready; its commit also covers PV_x(j-1): P buffer free, O quiescent
        ok = __all_sync(0xffffffffu, mbar_wait(bar(S_FULL_A + x), ph & 1, abort_flag, a.status));
        if (!ok) break;
        tc_fence_after();
        uint32_t r32[128];
        const bool masked = (a.causal && j == nt - 1) || j * BN + BN > a.seq_len;
        const int key_lim = min(a.seq_len, a.causal ? q_idx + 1 : a.seq_len) - j * BN;  // live keys [0, key_lim)
        // S_x(j) columns [64 h0, 64 h1) -> r32, keys past key_lim -> -inf
        auto load_s = [&](int h0, int h1) {
#pragma unroll
          for (int c = 2 * h0; c < 2 * h1; ++c)
            tmem_ld32(lane_base + s_col + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&r32[c * 32]));
          tmem_wait_ld();
          if (masked) {
#pragma unroll
            for (int i = 64 * h0; i < 64 * h1; ++i)
              if (i >= key_lim) r32[i] = __float_as_uint(-INFINITY);
          }
        };
        load_s(0, 2);
        // p = 2^(s * scale * log2e - m) for keys [64 hh, 64 hh + 64): one packed
        // FFMA per two scores and one MUFU.EX2 per score, row sums in s2, f16
        // pairs in w[hh]
        const float2 sc2 = make_float2(a.scale_log2, a.scale_log2);
        float2 s2[4];
        uint32_t w[2][32];
        auto exps = [&](int hh, float neg_m) {
          const float2 nm2 = make_float2(neg_m, neg_m);
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const int i = hh * 64 + 2 * e;
            const float2 xx = ffma2(make_float2(__uint_as_float(r32[i]), __uint_as_float(r32[i + 1])), sc2, nm2);
            const float p0 = ex2(xx.x);
            const float p1 = ex2(xx.y);
            s2[e & 3] = fadd2(s2[e & 3], make_float2(p0, p1));
            w[hh][e] = pack_half2(p0, p1);
          }
        };
#pragma unroll
        for (int i = 0; i < 4; ++i) s2[i] = make_float2(0.0f, 0.0f);
        // row max of the 128 scores: three-input max, four independent chains
        float mx[4];
        auto max_half = [&](int hh) {
#pragma unroll
          for (int i = hh * 64; i < hh * 64 + 64; i += 2)
            mx[(i >> 1) & 3] = fmax3(mx[(i >> 1) & 3], __uint_as_float(r32[i]), __uint_as_float(r32[i + 1]));
        };
#pragma unroll
        for (int i = 0; i < 4; ++i) mx[i] = -INFINITY;
        float m_new, corr, neg_m;
        bool any_grow;
        // the tile's row max -> the running max m_new (raised only when the
        // max grows by more than 2^8), the O / l correction and -m_new
        auto settle = [&]() {
          const float m_raw = fmax3(fmax3(mx[0], mx[1], mx[2]), mx[3], -INFINITY);
          const float m_t = m_raw == -INFINITY ? -INFINITY : m_raw * a.scale_log2;
          const bool grow = m_t > m_used + 8.0f;
          m_new = grow ? m_t : m_used;
          corr = (grow && m_used != -INFINITY) ? ex2(m_used - m_new) : 1.0f;
          neg_m = m_new == -INFINITY ? 0.0f : -m_new;
          any_grow = __any_sync(0xffffffffu, grow);
        };
        // the running max rose by more than 2^8: rescale this row of O
        // (quiescent: S_x(j)'s commit covered PV_x(j-1), and no MMA of
        // PV_x(j) starts before this warp's P_HALF arrival below)
        auto rescale_o = [&]() {
#pragma unroll 1
          for (int c = 0; c < 8; ++c) {  // 16 columns at a time
            uint32_t o[16];
            tmem_ld16(lane_base + o_col + c * 16, o);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 16; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * corr);
            tmem_st16(lane_base + o_col + c * 16, o);
          }
        };
        if (__all_sync(0xffffffffu, m_used != -INFINITY)) {
          // Every row of the warp has a running max (after the item's first
          // key tile): keys [0, 64) are exponentiated against it while the
          // tile's max is still being reduced.  A row whose max rises by more
          // than 2^8 is recomputed (its S columns reloaded from TMEM, where P
          // has not been written yet); every other row keeps m_used, exactly
          // as if the max had come first, so the results do not depend on the
          // speculation.
          max_half(0);  // issued first so that keys [0, 64) die with their exponentials
          exps(0, -m_used);
          max_half(1);
          settle();
          if (any_grow) {
            rescale_o();
            load_s(0, 1);
#pragma unroll
            for (int i = 0; i < 4; ++i) s2[i] = make_float2(0.0f, 0.0f);
            exps(0, neg_m);
          }
        } else {
          max_half(0);
          max_half(1);
          settle();
          if (j > 0 && any_grow) rescale_o();
          exps(0, neg_m);
        }
        // keys [0, 64) of P are published on P_HALF_x as soon as they have
        // landed, so the tensor core runs the first half of PV_x(j) while
        // keys [64, 128) are exponentiated
        tmem_st32(lane_base + s_col, w[0]);
        tmem_wait_st();  // keys [0, 64) of P (and any O rescale) have landed
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(P_HALF_A + x));
        exps(1, neg_m);
        tmem_st32(lane_base + s_col + 32, w[1]);
        tmem_wait_st();  // keys [64, 128) of P have landed
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(P_FULL_A + x));
        const float2 s4 = fadd2(fadd2(s2[0], s2[1]), fadd2(s2[2], s2[3]));
        l = l * corr + (s4.x + s4.y);
        m_used = m_new;
      }
      if (!ok) break;
      // the row sum goes to the epilogue warps through shared memory (two
      // slots: item n's slot is reused by item n + 2, whose last P cannot be
      // stored before item n's epilogue has handed O_x back)
      l_sm[(x * 2 + (nitems & 1)) * 128 + row] = l;
      ++nitems;
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(L_READY_A + x));
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem), "r"(kTmemCols));
  }
}

}  // namespace pf

// ---- host -----------------------------------------------------------------
namespace {

// [rows, heads, 128] f16 viewed as a 3-D tensor {128, heads, rows}; boxes of
// 64 x 1 x box_rows elements with the 128-byte swizzle.
int make_map(CUtensorMap* m, const void* base, uint64_t rows, uint64_t heads, uint32_t box_rows) {
  return encode_rows_map(m, base, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, 128, heads, rows, 64, box_rows,
                         "prefill");
}

}  // namespace

int launch_prefill_f16(const void* q, const void* k, const void* v, float* out, uint32_t seq_len,
                       uint32_t num_heads, uint32_t num_kv_heads, float scale, uint32_t causal,
                       const doe_paged_kv* cache, uint32_t cache_seq, uint32_t cache_start,
                       const doe_launch* launch) {
  int rc = DOE_OK;
  for (const void* p : {q, k, v, (const void*)out})
    if (reinterpret_cast<uintptr_t>(p) % 16 != 0) {
      set_op_error("prefill: q, k, v and out must be 16-byte aligned");
      return DOE_INVALID_ARGUMENT;
    }
  CUtensorMap mq, mk, mv, mck, mcv, mo;
  rc = make_map(&mq, q, seq_len, num_heads, 128);
  if (rc == DOE_OK) rc = make_map(&mk, k, seq_len, num_kv_heads, 128);
  if (rc == DOE_OK) rc = make_map(&mv, v, seq_len, num_kv_heads, 128);
  // f32 output rows [S, H, 128]: boxes of 32 columns x 32 rows (128-byte rows)
  if (rc == DOE_OK)
    rc = encode_rows_map(&mo, out, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, 128, num_heads, seq_len, 32, 32,
                         "prefill");
  pf::Args a;
  a.out = out;
  a.status = launch->status;
  a.table = nullptr;
  a.seq_len = (int)seq_len;
  a.num_heads = (int)num_heads;
  a.num_kv_heads = (int)num_kv_heads;
  a.n_qtiles = (int)((seq_len + 127) / 128);
  a.n_pairs = (a.n_qtiles + 1) / 2;
  a.causal = causal ? 1 : 0;
  a.cache_page_size = a.cache_num_pages = a.cache_max_pages = a.cache_start = 0;
  a.scale_log2 = scale * kLog2e;
  if (rc == DOE_OK && cache != nullptr) {
    const uint64_t rows = (uint64_t)cache->num_pages * cache->page_size;
    rc = make_map(&mck, cache->k_pool, rows, cache->num_kv_heads, 16);
    if (rc == DOE_OK) rc = make_map(&mcv, cache->v_pool, rows, cache->num_kv_heads, 16);
    a.table = cache->block_table + (size_t)cache_seq * cache->max_pages_per_seq;
    a.cache_page_size = (int)cache->page_size;
    a.cache_num_pages = (int)cache->num_pages;
    a.cache_max_pages = (int)cache->max_pages_per_seq;
    a.cache_start = (int)cache_start;
  } else {
    mck = mk;
    mcv = mv;
  }
  if (rc != DOE_OK) return rc;
  static std::atomic<bool> attr_set[kMaxDevices];
  rc = once_per_device(attr_set, [] {
    return cuda_status(cudaFuncSetAttribute(pf::prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            pf::kSmemBytes),
                       "cudaFuncSetAttribute(prefill)");
  });
  if (rc != DOE_OK) return rc;
  // persistent: one CTA per SM walks its zig-zag list of (pair, head) items
  const uint64_t items = (uint64_t)a.n_pairs * num_heads;
  a.num_items = (int)items;
  const uint64_t ctas = items < (uint64_t)num_sms() ? items : (uint64_t)num_sms();
  pf::prefill_kernel<<<(unsigned)ctas, pf::kThreads, pf::kSmemBytes,
                       static_cast<cudaStream_t>(launch->stream)>>>(mq, mk, mv, mck, mcv, mo, a);
  return cuda_status(cudaGetLastError(), "prefill_kernel");
}

}  // namespace doe
