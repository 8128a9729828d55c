// paged_decode.cu -- batched GQA decode over a paged KV cache (f16 or int8),
// split-K over the KV length with the splits stitched by the last CTA of each
// (sequence, kv head) to finish, fused new-token append.  Also the combine
// kernel of the f32 decode's many-split path (launch_combine_natural).
//
// Semantics: attention_head256_f16kv.wgsl with query_len 1 (every key of the
// sequence active), GQA kv_head = h / (H / Hkv) (…wgsl:46-49), paged rows
// phys = table[p / page] * page + p % page (…wgsl:51-63), out = acc / l or 0
// when l == 0 (…wgsl:257-268); split partials stitched with the log-sum-exp
// recipe of bench/tools/attention_kv_axis_sharded_stitch.py:46-90.
//
// Design (B200): the work is HBM-bound (2 flop/byte), so the kernel is built
// around the loads.  One warp consumes one 16-token tile (a page, or a
// 16-token slice of a larger page) per step.  Each warp has its own ring of
// tiles filled by TMA (one elected lane issues the boxes, an mbarrier per
// slot): the copies bypass the load/store pipe, which is left to the
// fragment reads.  Boxes land with the 128-byte swizzle, so the 16-byte
// fragment reads of a warp are conflict-free.  A dimension permutation,
// applied identically to Q, makes each lane's fragment bytes contiguous.
//   S  = Q K^T   : m16n8k16, rows = the GROUP query heads of one kv head
//   O^T = V^T P^T: m16n8k16, rows = 16 head dims, cols = the GROUP heads
// so P moves from the S accumulator into the PV B operand without shuffles.
// int8 tiles convert exactly to f16 in registers as 1152 + b (the byte, sign
// flipped, in the low half of 1024's f16 bits); the 1152 offsets are removed
// once per row instead of per element: S -= 1152 * sum(q), O -= 1152 *
// sum(f16 P).  The K scale multiplies S and the V scale folds into P.  Scores
// run in the log2 domain (the SFU's ex2 per key; exp2f for the merges).
// Prologue: each warp's page ids go to shared memory and its first copy is
// issued before the query work (before griddepcontrol.wait when the caller
// sets DOE_DECODE_INPUTS_STABLE); the warp whose walk holds the new row's
// tile appends the row, so no other warp waits for it.
#include "tma.cuh"

namespace doe {

struct PagedDecodeArgs {
  const __half* q;          // [B, H, D]
  const uint8_t* k_pool;    // [rows, Hkv, D] f16 or int8
  const uint8_t* v_pool;
  const __half* k_scale;    // [num_pages, Hkv, page_size] (int8 only)
  const __half* v_scale;
  const int32_t* block_table;  // [B, max_pages]
  const int32_t* seq_lens;     // [B]
  const __half* new_k;      // [B, Hkv, D] or null
  const __half* new_v;
  float* out;               // [B, H, D] f32, or bf16 storage when out_bf16
  float* part_o;            // [B*Hkv*max_splits, GROUP, D]
  float* part_ml;           // [B*Hkv*max_splits, GROUP, 2]
  unsigned* counters;       // [B*Hkv] arrivals per (b, g); zero at launch, left zero by the stitch
  int32_t* status;
  const float* freq_cis;    // RoPE table [rope_positions, D/2, {cos, sin}] or null
  int rope_positions;
  int window;               // > 0: only the last `window` keys attend
  float softcap;            // > 0: s = softcap * tanh(s / softcap) on the scaled score
  float scale;              // the natural-domain scale (softcap path)
  int num_heads, num_kv_heads, num_pages, page_size, max_pages;
  int split_tiles, max_splits;
  int out_bf16;
  float scale_log2;
  int page_shift;           // log2(page_size) when it is a power of two, else -1
  int inputs_stable;        // DOE_DECODE_INPUTS_STABLE: first copies before griddepcontrol.wait
};

// pos / page_size: a shift for power-of-two pages (every common size), so the
// per-tile copy issue carries no integer division
__device__ __forceinline__ int page_of(const PagedDecodeArgs& a, int pos) {
  return a.page_shift >= 0 ? pos >> a.page_shift : pos / a.page_size;
}

constexpr int kD = 128;
constexpr int kWarps = 4;
constexpr int kPageRegs = 4;  // page ids per lane at the prologue: 128 tiles per warp, 512 per split

__device__ __forceinline__ uint4 ldcg4(const uint8_t* p) {
  uint4 v;
  asm volatile("ld.global.cg.v4.u32 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ uint32_t w4(const uint4& v, int i) {
  return i == 0 ? v.x : (i == 1 ? v.y : (i == 2 ? v.z : v.w));
}

// Clamped sequence length and split count, shared with the combine kernel.
__device__ __forceinline__ int clamp_len(int len, int cap) {
  return len < 0 ? 0 : (len > cap ? cap : len);
}

// The new token's K/V row of kv head g at position pos, written by one warp
// in two steps: load() fetches the f16 rows (and the RoPE factors) right after
// the launch's wait, store() rotates, quantises and writes them into the pool
// later, when the loads have landed, so neither stalls the warp's walk.
template <bool INT8>
struct AppendRow {
  uint2 raw[2];       // lane's 4 elements of the K and the V row
  float rc[4], rsn[4];
  int page, in_page;

  __device__ __forceinline__ void load(const PagedDecodeArgs& a, int b, int g, int pos, const int32_t* table,
                                       int lane) {
    const int pidx = pos / a.page_size;
    page = table[pidx];
    in_page = pos - pidx * a.page_size;
    const size_t src = ((size_t)b * a.num_kv_heads + g) * kD + 4 * lane;  // lane owns [4 lane, 4 lane + 4)
    raw[0] = *reinterpret_cast<const uint2*>(a.new_k + src);
    raw[1] = *reinterpret_cast<const uint2*>(a.new_v + src);
    // RoPE on the K row: dim d < 64 (lanes 0-15) pairs with d + 64 (lane ^ 16)
    if (a.freq_cis != nullptr)
      rope_table<2>(a.freq_cis, a.rope_positions, kD / 2, pos, 4 * (lane & 15), a.status, lane == 0, rc, rsn);
  }

  // Ends with the fence that lets this warp's later TMA copies (the async
  // proxy) read the row.
  __device__ __forceinline__ void store(const PagedDecodeArgs& a, int g, int lane) {
    if ((unsigned)page >= (unsigned)a.num_pages) {
      if (lane == 0) report(a.status, DOE_DEVICE_ERR_PAGE);
      return;
    }
    const size_t row = (size_t)page * a.page_size + in_page;
    const int Hkv = a.num_kv_heads;
    const uint8_t* pools[2] = {a.k_pool, a.v_pool};
    const __half* scales[2] = {a.k_scale, a.v_scale};
#pragma unroll
    for (int kv = 0; kv < 2; ++kv) {
      uint2 v = raw[kv];
      if (kv == 0 && a.freq_cis != nullptr) {
        const uint2 partner = make_uint2(__shfl_xor_sync(0xffffffffu, v.x, 16), __shfl_xor_sync(0xffffffffu, v.y, 16));
        rope_rotate<2>(reinterpret_cast<const uint32_t*>(&raw[0]), reinterpret_cast<const uint32_t*>(&partner),
                       lane < 16, rc, rsn, reinterpret_cast<uint32_t*>(&v));
      }
      if (!INT8) {
        uint8_t* dst = const_cast<uint8_t*>(pools[kv]) + (row * Hkv + g) * (kD * 2) + 8 * lane;
        *reinterpret_cast<uint2*>(dst) = v;
      } else {
        __half2 h01 = *reinterpret_cast<__half2*>(&v.x);
        __half2 h23 = *reinterpret_cast<__half2*>(&v.y);
        float x[4] = {__low2float(h01), __high2float(h01), __low2float(h23), __high2float(h23)};
        float amax = fmaxf(fmaxf(fabsf(x[0]), fabsf(x[1])), fmaxf(fabsf(x[2]), fabsf(x[3])));
        amax = warp_max(amax);
        __half sh = __float2half_rn(div127(amax));
        float sf = __half2float(sh);
        int qv[4] = {0, 0, 0, 0};
        if (sf != 0.0f) {
          const float rs = __frcp_rn(sf);
#pragma unroll
          for (int e = 0; e < 4; ++e) qv[e] = quantize_s8(x[e], sf, rs);
        }
        const uint32_t packed = pack_s8x4(qv[0], qv[1], qv[2], qv[3]);
        uint8_t* dst = const_cast<uint8_t*>(pools[kv]) + (row * Hkv + g) * kD + 4 * lane;
        *reinterpret_cast<uint32_t*>(dst) = packed;
        if (lane == 0) {
          __half* sdst = const_cast<__half*>(scales[kv]);
          sdst[((size_t)page * Hkv + g) * a.page_size + in_page] = sh;
        }
      }
    }
    asm volatile("fence.proxy.async.global;\n" ::: "memory");
    __syncwarp();
  }
};

// Per-warp ring of TMA-filled tiles.  A slot holds one 16-token tile, each
// 16-row x 128-byte box on a 1024-byte boundary (chunk x of row R at x ^ R%8):
//   f16:  K dims 0-63 | K dims 64-127 | V dims 0-63 | V dims 64-127   (8 KB)
//   int8: K (128 dims) | V (128 dims)                                  (4 KB)
// int8 slots also take the tile's 16 K scales and 16 V scales (64 B, kept
// after the tiles).  Slot reuse is ordered by the warp itself: it issues the
// refill of a slot only after it has read the slot's previous tile.
template <bool INT8>
struct Ring {
  static constexpr int kStages = 2;
  static constexpr int kTile = INT8 ? 4096 : 8192;
  static constexpr int kScale = INT8 ? 64 : 0;
  static constexpr int kTx = kTile + kScale;                       // bytes per filled slot
  static constexpr int kWarpBytes = (kStages * (kTile + kScale) + 1023) / 1024 * 1024;
  static constexpr int kSmem = kWarps * kWarpBytes + 1024;         // + base alignment
};

__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr));
  return v;
}
__device__ __forceinline__ uint32_t lds32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];\n" : "=r"(v) : "r"(addr));
  return v;
}

// 2^x on the SFU (ex2.approx.ftz: relative error ~2^-22, -inf -> +0), for the
// per-key exponentials of the online softmax
__device__ __forceinline__ float ex2a(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;\n" : "=f"(y) : "f"(x));
  return y;
}
// CAP: the score softcap is compiled in only where a launch asks for it
template <bool INT8, int GROUP, bool CAP>
__global__ void __launch_bounds__(kWarps * 32)
    paged_decode_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                        const PagedDecodeArgs a) {
  using R = Ring<INT8>;
  constexpr int P = R::kStages;
  extern __shared__ __align__(1024) uint8_t dsmem_raw[];
  // the swizzled boxes need 1024-byte alignment
  uint8_t* dsmem = dsmem_raw + ((1024 - (smem_addr(dsmem_raw) & 1023)) & 1023);
  // launched with launch_pdl: q, new K/V and (unless inputs_stable) the
  // lengths, table and pools come from earlier kernels
  if (!a.inputs_stable) pdl_wait();
  const int split = blockIdx.x, g = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = lane >> 2, c = lane & 3;
  const int Hkv = a.num_kv_heads;

  const int raw_len = a.seq_lens[b];
  const int cap = a.max_pages * a.page_size;
  const int seq_len = clamp_len(raw_len, cap);
  if (raw_len != seq_len && split == 0 && g == 0 && threadIdx.x == 0)
    report(a.status, DOE_DEVICE_ERR_LENGTH);
  // sliding window (attention_head256_f16kv.wgsl:129-135 at abs_q = seq_len - 1):
  // keys [min_key, seq_len); the tiles start at the one holding min_key
  const int min_key = (a.window > 0 && seq_len > a.window) ? seq_len - a.window : 0;
  const int tile_origin = min_key >> 4;
  const int ntiles = ((seq_len + 15) >> 4) - tile_origin;
  const int nsplits = max(1, (ntiles + a.split_tiles - 1) / a.split_tiles);
  if (split >= nsplits) return;
  const int tile_begin = split * a.split_tiles;  // relative to tile_origin
  const int tile_end = min(ntiles, tile_begin + a.split_tiles);
  const int32_t* table = a.block_table + (size_t)b * a.max_pages;

  __shared__ float sm_m[kWarps][8];
  __shared__ float sm_l[kWarps][8];
  __shared__ int sm_last;
  __shared__ int sm_pg[kWarps][32 * kPageRegs];
  __shared__ __align__(8) uint64_t ring_bar[kWarps][P];

  if (lane == 0) {
#pragma unroll
    for (int st = 0; st < P; ++st) mbar_init(smem_addr(&ring_bar[warp][st]), 1);
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  __syncwarp();

  // ---- this warp's tiles: tile_begin + warp + 4k, k < nt; page ids up front
  const int span = tile_end - tile_begin - warp;
  const int nt = span > 0 ? (span + kWarps - 1) / kWarps : 0;
  // page ids of the warp's tiles, one shared-memory word per tile (one load
  // per lookup, as cheap as a shuffle, for any number of tiles up to the cap)
#pragma unroll
  for (int i = 0; i < kPageRegs; ++i)
    if (lane + 32 * i < nt)
      sm_pg[warp][lane + 32 * i] = table[page_of(a, (tile_origin + tile_begin + warp + kWarps * (lane + 32 * i)) << 4)];
  __syncwarp();
  auto page_of_tile = [&](int k) { return sm_pg[warp][k]; };  // k < nt

  const int vt[4] = {2 * c, 2 * c + 1, 2 * c + 8, 2 * c + 9};
  const uint32_t wbase = smem_addr(dsmem) + warp * R::kWarpBytes;
  auto slot = [&](int k) { return wbase + (k % P) * R::kTile; };
  auto scales = [&](int k) { return wbase + P * R::kTile + (k % P) * R::kScale; };

  // Fills slot k % P with tile k (whole warp calls, one lane issues).  A tile
  // whose page id is out of range gets a plain arrival instead, so the slot's
  // barrier phase still advances; the consumer reports the bad page.
  auto issue = [&](int k) {
    const int page = page_of_tile(k);
    if (lane != 0) return;
    const uint32_t bar = smem_addr(&ring_bar[warp][k % P]);
    if ((unsigned)page >= (unsigned)a.num_pages) {
      mbar_arrive(bar);
      return;
    }
    const int pos0 = (tile_origin + tile_begin + warp + kWarps * k) << 4;
    const int pidx = page_of(a, pos0);
    const int in0 = pos0 - pidx * a.page_size;
    const int row0 = page * a.page_size + in0;
    const uint32_t dst = slot(k);
    // this warp read the slot's previous tile through the generic proxy
    asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
    mbar_expect_tx(bar, R::kTx);
    if (!INT8) {
      tma_load_3d(dst, &tm_k, bar, 0, g, row0);
      tma_load_3d(dst + 2048, &tm_k, bar, 64, g, row0);
      tma_load_3d(dst + 4096, &tm_v, bar, 0, g, row0);
      tma_load_3d(dst + 6144, &tm_v, bar, 64, g, row0);
    } else {
      tma_load_3d(dst, &tm_k, bar, 0, g, row0);
      tma_load_3d(dst + 2048, &tm_v, bar, 0, g, row0);
      const size_t sidx = ((size_t)page * Hkv + g) * a.page_size + in0;
      bulk_load(scales(k), a.k_scale + sidx, 32, bar);
      bulk_load(scales(k) + 32, a.v_scale + sidx, 32, bar);
    }
  };

  // The first copies of the ring go out before the query work, and before
  // griddepcontrol.wait when the caller vouches that seq_lens, the block table
  // and the pool rows are final (DOE_DECODE_INPUTS_STABLE); a tile holding the
  // row this launch appends waits for the append.
  const bool appends = a.new_k != nullptr && split == nsplits - 1 && seq_len > 0;
  const int new_tile = ((seq_len - 1) >> 4) - tile_origin - tile_begin;  // split-relative
  int issued = 0;
  for (; issued < P - 1 && issued < nt; ++issued)
    if (appends && new_tile == warp + kWarps * issued) break;
    else issue(issued);
  if (a.inputs_stable) pdl_wait();
  pdl_trigger();

  // the warp whose walk holds the new row's tile appends the row itself, so
  // no other warp waits for it: loads now, the pool write after the query's
  // loads, before any copy of that tile
  const bool append_pending = appends && new_tile % kWarps == warp;
  AppendRow<INT8> app;
  if (append_pending) app.load(a, b, g, seq_len - 1, table, lane);

  // ---- Q fragments (rows = heads g*GROUP + r, r < GROUP) -----------------
  // f16 pools:  k-block j = 2i + jj holds dims 32i + 8c + 4jj + {0,1 | 2,3}
  // int8 pools: k-block j = 4i + w  holds dims 64i + 16c + 4w + {0,1 | 2,3}
  uint32_t qa[8][2];
  {
    const __half* qrow = a.q + ((size_t)b * a.num_heads + (size_t)g * GROUP + r) * kD;
    const bool live = r < GROUP;
    // the lane's four 8-dim runs: index 2i + part (int8) or i (f16); runs 0, 1
    // lie in the first half of the head dims and runs 2, 3 hold their RoPE
    // partners 64 dims on
    uint4 qv[4];
#pragma unroll
    for (int n = 0; n < 4; ++n) {
      const int dim0 = INT8 ? (64 * (n >> 1) + 16 * c + 8 * (n & 1)) : (32 * n + 8 * c);
      qv[n] = live ? *reinterpret_cast<const uint4*>(qrow + dim0) : make_uint4(0, 0, 0, 0);
    }
    if (a.freq_cis != nullptr && live && seq_len > 0) {
      // the query sits at the new token's position, seq_len - 1
#pragma unroll
      for (int n = 0; n < 2; ++n) {
        float rc[8], rsn[8];
        const int pair0 = INT8 ? (16 * c + 8 * n) : (32 * n + 8 * c);
        rope_table<4>(a.freq_cis, a.rope_positions, kD / 2, (long long)seq_len - 1, pair0, a.status,
                      split == 0 && g == 0 && r == 0 && c == 0 && warp == 0, rc, rsn);
        const uint4 lo = qv[n], hi = qv[n + 2];
        rope_rotate<4>(reinterpret_cast<const uint32_t*>(&lo), reinterpret_cast<const uint32_t*>(&hi), true, rc,
                       rsn, reinterpret_cast<uint32_t*>(&qv[n]));
        rope_rotate<4>(reinterpret_cast<const uint32_t*>(&hi), reinterpret_cast<const uint32_t*>(&lo), false, rc,
                       rsn, reinterpret_cast<uint32_t*>(&qv[n + 2]));
      }
    }
#pragma unroll
    for (int i = 0; i < (INT8 ? 2 : 4); ++i) {
#pragma unroll
      for (int part = 0; part < (INT8 ? 2 : 1); ++part) {
        const uint4 v = qv[INT8 ? 2 * i + part : i];
        if (!INT8) {
          qa[2 * i][0] = v.x; qa[2 * i][1] = v.y;
          qa[2 * i + 1][0] = v.z; qa[2 * i + 1][1] = v.w;
        } else {
          // 8 dims = words 2w', 2w'+1 of the 16-dim run; k-block 4i + w
          const int w0 = 2 * part;
          qa[4 * i + w0][0] = v.x; qa[4 * i + w0][1] = v.y;
          qa[4 * i + w0 + 1][0] = v.z; qa[4 * i + w0 + 1][1] = v.w;
        }
      }
    }
  }

  // int8: 1152 * sum of this row's query (its 32 dims per lane, then the 4
  // lanes of the row), taken off every score
  float q1152 = 0.0f;
  if (INT8) {
    float qs = 0.0f;
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
      for (int w = 0; w < 2; ++w) {
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&qa[j][w]));
        qs += f.x + f.y;
      }
    qs += __shfl_xor_sync(0xffffffffu, qs, 1);
    qs += __shfl_xor_sync(0xffffffffu, qs, 2);
    q1152 = 1152.0f * qs;
  }
  float p1152 = 0.0f;  // int8: running sum of this row's f16 P (times 1152 at the end)


  float m_run = -INFINITY, l_run = 0.0f;
  float acc[8][4];
#pragma unroll
  for (int mb = 0; mb < 8; ++mb) acc[mb][0] = acc[mb][1] = acc[mb][2] = acc[mb][3] = 0.0f;

  // after the query's loads: the row's loads, issued with them, have landed
  if (append_pending) app.store(a, g, lane);
  for (int s0 = issued; s0 < P - 1; ++s0)
    if (s0 < nt) issue(s0);
  bool ring_ok = true;
  for (int k = 0; k < nt; ++k) {
    if (k + P - 1 < nt) issue(k + P - 1);
    // tile k has landed (bounded: a timeout ends this warp's walk)
    ring_ok = __all_sync(0xffffffffu, mbar_wait_bounded(smem_addr(&ring_bar[warp][k % P]), (k / P) & 1));
    if (!ring_ok) {
      if (lane == 0) report(a.status, DOE_DEVICE_ERR_TIMEOUT);
      break;
    }
    const int page = page_of_tile(k);
    if ((unsigned)page >= (unsigned)a.num_pages) {
      if (lane == 0) report(a.status, DOE_DEVICE_ERR_PAGE);
      continue;
    }
    const int pos0 = (tile_origin + tile_begin + warp + kWarps * k) << 4;
    const uint32_t sb = slot(k);

    // Fragment reads (swizzled chunk positions; see Ring).  K: lane (r, c)
    // takes row nb*8 + r, 16-byte chunk 4*(i&1) + c of box i>>1 (f16) or
    // chunk 4i + c (int8).  V: row vt[j], chunk r of box h.
    uint4 kraw[2][INT8 ? 2 : 4];
    uint4 vraw[4][INT8 ? 1 : 2];
#pragma unroll
    for (int nb = 0; nb < 2; ++nb)
#pragma unroll
      for (int i = 0; i < (INT8 ? 2 : 4); ++i) {
        const int box = INT8 ? 0 : (i >> 1), chunk = INT8 ? (4 * i + c) : (4 * (i & 1) + c);
        kraw[nb][i] = lds128(sb + box * 2048 + (nb * 8 + r) * 128 + ((chunk ^ r) << 4));
      }
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int h = 0; h < (INT8 ? 1 : 2); ++h)
        vraw[j][h] = lds128(sb + (INT8 ? 2048 : 4096 + h * 2048) + vt[j] * 128 + ((r ^ (vt[j] & 7)) << 4));
    uint32_t ksc[2] = {0, 0}, vsc[2] = {0, 0};
    if (INT8) {
      const uint32_t ss = scales(k);
      ksc[0] = lds32(ss + 4 * c);        // tokens 2c, 2c+1
      ksc[1] = lds32(ss + 16 + 4 * c);   // tokens 8+2c, 9+2c
      vsc[0] = lds32(ss + 32 + 4 * c);
      vsc[1] = lds32(ss + 48 + 4 * c);
    }

    // ---- S = Q K^T ----------------------------------------------------------
    float s[2][4];
#pragma unroll
    for (int nb = 0; nb < 2; ++nb) {
      s[nb][0] = s[nb][1] = s[nb][2] = s[nb][3] = 0.0f;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        uint32_t b0, b1;
        if (!INT8) {
          const uint4& v = kraw[nb][j >> 1];
          b0 = w4(v, 2 * (j & 1));
          b1 = w4(v, 2 * (j & 1) + 1);
        } else {
          // bytes 0,1 / 2,3 -> f16 halves 1152 + k: sign-flipped byte under 0x64
          const uint32_t x = w4(kraw[nb][j >> 2], j & 3) ^ 0x80808080u;
          b0 = prmt(x, 0x64646464u, 0x4140);
          b1 = prmt(x, 0x64646464u, 0x4342);
        }
        mma_16816(s[nb], qa[j][0], 0u, qa[j][1], 0u, b0, b1);
      }
    }

    // ---- online softmax (log2 domain), rows r ------------------------------
    float x[2][2];
    // only the window's first tile and the sequence's last hold dead keys;
    // int8 tiles skip the per-key checks elsewhere (the f16 kernel, bound by
    // HBM rather than issue, keeps them)
    const bool edge = !INT8 || pos0 < min_key || pos0 + 16 > seq_len;
#pragma unroll
    for (int nb = 0; nb < 2; ++nb) {
      // the two keys of a score pair in packed FP32: (s - 1152 sum q) * k_scale,
      // then the log2-domain scale, each product and sum rounded as in scalar form
      float2 sv = make_float2(s[nb][0], s[nb][1]);
      if (INT8)
        sv = fmul2(fadd2(sv, make_float2(-q1152, -q1152)),
                   __half22float2(*reinterpret_cast<const __half2*>(&ksc[nb])));
      if (CAP) {
        // softcap (…wgsl:197-199): cap * tanh((q.k * scale) / cap), then log2 domain
        x[nb][0] = a.softcap * tanhf(sv.x * a.scale / a.softcap) * kLog2e;
        x[nb][1] = a.softcap * tanhf(sv.y * a.scale / a.softcap) * kLog2e;
      } else {
        const float2 xs = fmul2(sv, make_float2(a.scale_log2, a.scale_log2));
        x[nb][0] = xs.x;
        x[nb][1] = xs.y;
      }
    }
    if (edge) {
#pragma unroll
      for (int nb = 0; nb < 2; ++nb)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int key = pos0 + nb * 8 + 2 * c + e;
          if (!(key < seq_len && key >= min_key)) x[nb][e] = -INFINITY;
        }
    }
    float tmax = fmaxf(fmaxf(x[0][0], x[0][1]), fmaxf(x[1][0], x[1][1]));
    tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 1));
    tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 2));
    // lazy running max: it moves (and the accumulators are rescaled) only when
    // a row's max rises by more than 2^8, so p <= 256 (exact in f16 P) and
    // most tiles skip the rescale; the tile holds a valid key, so tmax is finite
    const bool grow = tmax > m_run + 8.0f;
    const float m_new = grow ? tmax : m_run;
    const float corr = grow ? ex2a(m_run - m_new) : 1.0f;
    float p[2][2];
#pragma unroll
    for (int nb = 0; nb < 2; ++nb)
#pragma unroll
      for (int e = 0; e < 2; ++e) p[nb][e] = ex2a(x[nb][e] - m_new);
    l_run = l_run * corr + ((p[0][0] + p[0][1]) + (p[1][0] + p[1][1]));
    m_run = m_new;

    float pv[2][2];
#pragma unroll
    for (int nb = 0; nb < 2; ++nb)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        float sc = 1.0f;
        if (INT8) {
          __half2 v2 = *reinterpret_cast<__half2*>(&vsc[nb]);
          sc = e ? __high2float(v2) : __low2float(v2);
        }
        pv[nb][e] = r < GROUP ? p[nb][e] * sc : 0.0f;  // dead keys have p = +0
      }
    const uint32_t pb0 = pack_half2(pv[0][0], pv[0][1]);
    const uint32_t pb1 = pack_half2(pv[1][0], pv[1][1]);
    if (INT8) {
      // the f16 P the PV product uses, summed for the 1152 offset of V
      const float2 f0 = __half22float2(*reinterpret_cast<const __half2*>(&pb0));
      const float2 f1 = __half22float2(*reinterpret_cast<const __half2*>(&pb1));
      p1152 = p1152 * corr + ((f0.x + f0.y) + (f1.x + f1.y));
    }

    if (__any_sync(0xffffffffu, grow)) {
      // accumulator columns are heads 2c, 2c+1: fetch their row corrections
      const float cA = __shfl_sync(0xffffffffu, corr, (2 * c) * 4);
      const float cB = __shfl_sync(0xffffffffu, corr, (2 * c + 1) * 4);
#pragma unroll
      for (int mb = 0; mb < 8; ++mb) {
        acc[mb][0] *= cA; acc[mb][2] *= cA;
        acc[mb][1] *= cB; acc[mb][3] *= cB;
      }
    }

    // f16 V rows past the sequence end may hold any bits: zero them
    if (!INT8) {
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (pos0 + vt[j] >= seq_len) vraw[j][0] = vraw[j][1] = make_uint4(0, 0, 0, 0);
    }

    // ---- O^T += V^T P^T ------------------------------------------------------
#pragma unroll
    for (int mb = 0; mb < 8; ++mb) {
      uint32_t a0, a1, a2, a3;
      if (!INT8) {
        // m-block mb = 4h + w: rows r / r+8 = dims 64h + 8r + 2w + {0 / 1}
        const int h = mb >> 2, w = mb & 3;
        const uint32_t x0 = w4(vraw[0][h], w), x1 = w4(vraw[1][h], w);
        const uint32_t x2 = w4(vraw[2][h], w), x3 = w4(vraw[3][h], w);
        a0 = prmt(x0, x1, 0x5410); a1 = prmt(x0, x1, 0x7632);
        a2 = prmt(x2, x3, 0x5410); a3 = prmt(x2, x3, 0x7632);
      } else {
        // m-block mb = 2w + e: rows r / r+8 = dims 16r + 4w + 2e + {0 / 1}
        const int w = mb >> 1, e = mb & 1;
        const uint32_t x0 = w4(vraw[0][0], w), x1 = w4(vraw[1][0], w);
        const uint32_t x2 = w4(vraw[2][0], w), x3 = w4(vraw[3][0], w);
        const uint32_t lo = e ? 0x0602u : 0x0400u, hi = e ? 0x0703u : 0x0501u;
        // f16 halves 1152 + v: (byte pair & 0x00ff00ff) ^ 0x64806480, one LOP3
        a0 = (prmt(x0, x1, lo) & 0x00ff00ffu) ^ 0x64806480u; a1 = (prmt(x0, x1, hi) & 0x00ff00ffu) ^ 0x64806480u;
        a2 = (prmt(x2, x3, lo) & 0x00ff00ffu) ^ 0x64806480u; a3 = (prmt(x2, x3, hi) & 0x00ff00ffu) ^ 0x64806480u;
      }
      mma_16816(acc[mb], a0, a1, a2, a3, pb0, pb1);
    }
  }

  if (INT8) {
    // O -= 1152 * sum(f16 P) per head: accumulator columns are heads 2c, 2c+1
    float ps = p1152;
    ps += __shfl_xor_sync(0xffffffffu, ps, 1);
    ps += __shfl_xor_sync(0xffffffffu, ps, 2);
    const float oA = 1152.0f * __shfl_sync(0xffffffffu, ps, (2 * c) * 4);
    const float oB = 1152.0f * __shfl_sync(0xffffffffu, ps, (2 * c + 1) * 4);
#pragma unroll
    for (int mb = 0; mb < 8; ++mb) {
      acc[mb][0] -= oA; acc[mb][2] -= oA;
      acc[mb][1] -= oB; acc[mb][3] -= oB;
    }
  }

  // ---- merge the warps of this split (O staged in this warp's own ring) ----
  l_run += __shfl_xor_sync(0xffffffffu, l_run, 1);
  l_run += __shfl_xor_sync(0xffffffffu, l_run, 2);
  if (c == 0 && r < GROUP) {
    sm_m[warp][r] = m_run;
    sm_l[warp][r] = l_run;
  }
  float* my_o = reinterpret_cast<float*>(dsmem + warp * R::kWarpBytes);  // [GROUP][kD]
#pragma unroll
  for (int mb = 0; mb < 8; ++mb) {
    const int d0 = INT8 ? (16 * r + 4 * (mb >> 1) + 2 * (mb & 1))
                        : (64 * (mb >> 2) + 8 * r + 2 * (mb & 3));
    if (2 * c < GROUP) {
      my_o[(2 * c) * kD + d0] = acc[mb][0];
      my_o[(2 * c) * kD + d0 + 1] = acc[mb][2];
    }
    if (2 * c + 1 < GROUP) {
      my_o[(2 * c + 1) * kD + d0] = acc[mb][1];
      my_o[(2 * c + 1) * kD + d0 + 1] = acc[mb][3];
    }
  }
  __syncthreads();

  const int dim = threadIdx.x;  // 128 threads == head dim
  float O[GROUP], L[GROUP], M[GROUP];
#pragma unroll
  for (int hh = 0; hh < GROUP; ++hh) {
    M[hh] = -INFINITY;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) M[hh] = fmaxf(M[hh], sm_m[w][hh]);
    O[hh] = 0.0f;
    L[hh] = 0.0f;
    if (M[hh] != -INFINITY) {
#pragma unroll
      for (int w = 0; w < kWarps; ++w) {
        const float f = exp2f(sm_m[w][hh] - M[hh]);  // -inf -> 0
        O[hh] += f * reinterpret_cast<const float*>(dsmem + w * R::kWarpBytes)[hh * kD + dim];
        L[hh] += f * sm_l[w][hh];
      }
    }
  }
  const size_t out_row = ((size_t)b * a.num_heads + (size_t)g * GROUP) * kD;
  auto store = [&](int hh, float v) {
    if (a.out_bf16)
      reinterpret_cast<__nv_bfloat16*>(a.out)[out_row + hh * kD + dim] = __float2bfloat16_rn(v);
    else
      a.out[out_row + hh * kD + dim] = v;
  };
  if (nsplits == 1) {
#pragma unroll
    for (int hh = 0; hh < GROUP; ++hh) store(hh, L[hh] > 0.0f ? O[hh] * (1.0f / L[hh]) : 0.0f);
    return;
  }
  // ---- split partials; the last split of (b, g) to finish stitches them ---
  const size_t base = ((size_t)b * Hkv + g) * a.max_splits;
#pragma unroll
  for (int hh = 0; hh < GROUP; ++hh) {
    const size_t prow = (base + split) * GROUP + hh;
    a.part_o[prow * kD + dim] = O[hh];
    if (dim == 0) {
      a.part_ml[prow * 2] = M[hh];
      a.part_ml[prow * 2 + 1] = L[hh];
    }
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned old = atomicAdd(&a.counters[(size_t)b * Hkv + g], 1u);
    sm_last = old == (unsigned)(nsplits - 1);
    if (sm_last) a.counters[(size_t)b * Hkv + g] = 0u;  // ready for the next launch
  }
  __syncthreads();
  if (!sm_last) return;
  __threadfence();
#pragma unroll
  for (int hh = 0; hh < GROUP; ++hh) {
    float MM = -INFINITY;
    for (int sp = 0; sp < nsplits; ++sp)
      MM = fmaxf(MM, __ldcg(a.part_ml + ((base + sp) * GROUP + hh) * 2));
    float OO = 0.0f, LL = 0.0f;
    if (MM != -INFINITY) {
      for (int sp = 0; sp < nsplits; ++sp) {
        const size_t prow = (base + sp) * GROUP + hh;
        const float f = exp2f(__ldcg(a.part_ml + prow * 2) - MM);
        OO += f * __ldcg(a.part_o + prow * kD + dim);
        LL += f * __ldcg(a.part_ml + prow * 2 + 1);
      }
    }
    store(hh, LL > 0.0f ? OO * (1.0f / LL) : 0.0f);
  }
}

// Stitches split partials: rows (b, kv head g, head-in-group hh).  Partial
// maxima are log2-domain when LOG2, natural otherwise.
struct CombineArgs {
  const float* part_o;
  const float* part_ml;
  float* out;
  const int32_t* seq_lens;  // null: every row has fixed_len tokens
  int fixed_len, cap, split_tokens, max_splits, num_kv_heads, group, head_dim;
};

template <bool LOG2>
__global__ void combine_splits_kernel(const CombineArgs a) {
  // all partial (max, sum) pairs of the row are fetched in parallel (one per
  // thread), weights computed once in shared memory, then every head dim
  // reads its split values with independent loads.
  __shared__ float w_sm[1024];
  __shared__ float inv_sm;
  const int h = blockIdx.x, b = blockIdx.y;
  const int g = h / a.group, hh = h - g * a.group;
  const int len = a.seq_lens ? clamp_len(a.seq_lens[b], a.cap) : a.fixed_len;
  const int nsplits = max(1, (len + a.split_tokens - 1) / a.split_tokens);
  if (nsplits == 1) return;  // the split kernel wrote the output
  const size_t base = ((size_t)b * a.num_kv_heads + g) * a.max_splits;
  const int tid = threadIdx.x;
  float m = -INFINITY, lsum = 0.0f;
  if (tid < nsplits) {
    const float* ml = a.part_ml + ((base + tid) * a.group + hh) * 2;
    m = ml[0];
    lsum = ml[1];
  }
  float M = m;
  for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
  __shared__ float wmax[32];
  if ((tid & 31) == 0) wmax[tid >> 5] = M;
  __syncthreads();
  M = -INFINITY;
  for (int i = 0; i < (int)(blockDim.x + 31) / 32; ++i) M = fmaxf(M, wmax[i]);
  const float f = (tid < nsplits && M != -INFINITY) ? (LOG2 ? exp2f(m - M) : expf(m - M)) : 0.0f;
  if (tid < nsplits) w_sm[tid] = f;
  float fl = f * lsum;
  for (int o = 16; o > 0; o >>= 1) fl += __shfl_xor_sync(0xffffffffu, fl, o);
  __syncthreads();
  if ((tid & 31) == 0) wmax[tid >> 5] = fl;
  __syncthreads();
  if (tid == 0) {
    float L = 0.0f;
    for (int i = 0; i < (int)(blockDim.x + 31) / 32; ++i) L += wmax[i];
    inv_sm = L > 0.0f ? 1.0f / L : 0.0f;
  }
  __syncthreads();
  const float inv = inv_sm;
  for (int d = tid; d < a.head_dim; d += blockDim.x) {
    float O = 0.0f;
    for (int sp = 0; sp < nsplits; ++sp)
      O += w_sm[sp] * a.part_o[((base + sp) * a.group + hh) * a.head_dim + d];
    a.out[((size_t)b * a.num_kv_heads * a.group + h) * a.head_dim + d] = O * inv;
  }
}

template __global__ void combine_splits_kernel<true>(const CombineArgs);
template __global__ void combine_splits_kernel<false>(const CombineArgs);

// ---------------------------------------------------------------------------
template <bool INT8, int GROUP, bool CAP>
static int launch_cap(const CUtensorMap& tm_k, const CUtensorMap& tm_v, const PagedDecodeArgs& a, dim3 grid,
                      cudaStream_t st) {
  constexpr int smem = Ring<INT8>::kSmem;
  static std::atomic<bool> attr[kMaxDevices];  // per instantiation and device
  const int rc = once_per_device(attr, [] {
    return cuda_status(cudaFuncSetAttribute(paged_decode_kernel<INT8, GROUP, CAP>,
                                            cudaFuncAttributeMaxDynamicSharedMemorySize, smem),
                       "cudaFuncSetAttribute(paged_decode)");
  });
  if (rc != DOE_OK) return rc;
  return cuda_status(
      launch_pdl(paged_decode_kernel<INT8, GROUP, CAP>, grid, dim3(kWarps * 32), smem, st, tm_k, tm_v, a),
      "paged_decode_kernel");
}

template <bool INT8, int GROUP>
static int launch_one(const CUtensorMap& tm_k, const CUtensorMap& tm_v, const PagedDecodeArgs& a, dim3 grid,
                      cudaStream_t st) {
  return a.softcap > 0.0f ? launch_cap<INT8, GROUP, true>(tm_k, tm_v, a, grid, st)
                          : launch_cap<INT8, GROUP, false>(tm_k, tm_v, a, grid, st);
}

int launch_paged_decode(const doe_paged_kv* kv, uint32_t num_seqs, uint32_t num_heads,
                        const void* q, const int32_t* seq_lens, const void* new_k,
                        const void* new_v, float scale, float* out, uint32_t split_pages,
                        const doe_decode_options* opts, const doe_launch* launch,
                        uint64_t* ws_needed_out) {
  const uint32_t Hkv = kv->num_kv_heads;
  const uint32_t group = num_heads / Hkv;
  const uint32_t tiles_per_page = kv->page_size / 16;
  const uint32_t max_tiles = kv->max_pages_per_seq * tiles_per_page;
  uint32_t split_tiles;
  if (split_pages) {
    split_tiles = split_pages * tiles_per_page;
  } else {
    // Long splits amortise each CTA's pipeline fill and stitch (64 tiles for
    // f16, 128 for int8 measured best on config 3 / 4, whose work fills
    // several waves of 3 CTAs per SM on 148 SMs at that length).  Less work
    // than that (a decode batch of uniform contexts, or one tensor-parallel
    // rank's few KV heads) gets as few splits as still keep about two CTAs
    // per SM busy, each at most 128 tiles and all of one length.  Where the
    // (sequence, kv head) rows alone put at least one CTA on every SM and fit
    // one wave of 3 per SM, and a row fits one split, each row is one split:
    // a second wave would start its CTAs while the first one's SMs idle on
    // their prologues (config 5: 256 rows, 0.778 -> 0.753 ms per step against
    // three splits in 1.7 waves).  Ragged lengths keep the short splits,
    // which balance as CTAs finish (config 4 split over 4 ranks: 16 splits of
    // 128 tiles, not 5 of 410).
    const uint64_t seq_rows = (uint64_t)num_seqs * Hkv;
    const uint64_t want = ((uint64_t)max_tiles * seq_rows + 1775) / 1776;
    const uint32_t cap = kv->kv_dtype == DOE_KV_INT8 ? 128u : 64u;
    const uint64_t sms = (uint64_t)num_sms();
    if (want >= cap) {
      split_tiles = cap;
    } else if (seq_rows >= sms && seq_rows <= 3 * sms && max_tiles <= (uint64_t)kWarps * 32 * kPageRegs) {
      split_tiles = max_tiles < 4 ? 4u : max_tiles;
    } else {
      uint64_t s = (max_tiles + 127) / 128;
      const uint64_t fill = (280 + seq_rows - 1) / seq_rows;
      if (s < fill) s = fill;
      if (s < 1) s = 1;
      const uint64_t t = (max_tiles + s - 1) / s;
      split_tiles = (uint32_t)(t < 4 ? 4 : t);
    }
  }
  if (split_tiles == 0) split_tiles = 1;
  if (split_tiles > kWarps * 32 * kPageRegs) split_tiles = kWarps * 32 * kPageRegs;  // prefetched page ids
  const uint32_t max_splits = max_tiles == 0 ? 1 : ceil_div(max_tiles, split_tiles);
  const uint64_t rows = (uint64_t)num_seqs * Hkv * max_splits * group;
  const uint64_t part_bytes = rows * (kD + 2) * sizeof(float);
  const uint64_t ctr_off = (part_bytes + 255) / 256 * 256;
  const uint64_t ws = ctr_off + (uint64_t)num_seqs * Hkv * sizeof(unsigned);
  if (ws_needed_out) {
    *ws_needed_out = ws;
    return DOE_OK;
  }
  if (launch->workspace == nullptr || launch->workspace_bytes < ws) {
    set_op_error("doe_paged_decode: workspace of %llu bytes required, %llu given",
                 (unsigned long long)ws, (unsigned long long)launch->workspace_bytes);
    return DOE_INVALID_ARGUMENT;
  }
  PagedDecodeArgs a;
  a.q = static_cast<const __half*>(q);
  a.k_pool = static_cast<const uint8_t*>(kv->k_pool);
  a.v_pool = static_cast<const uint8_t*>(kv->v_pool);
  a.k_scale = static_cast<const __half*>(kv->k_scale);
  a.v_scale = static_cast<const __half*>(kv->v_scale);
  a.block_table = kv->block_table;
  a.seq_lens = seq_lens;
  a.new_k = static_cast<const __half*>(new_k);
  a.new_v = static_cast<const __half*>(new_v);
  a.out = out;
  a.part_o = static_cast<float*>(launch->workspace);
  a.part_ml = a.part_o + rows * kD;
  a.counters = reinterpret_cast<unsigned*>(static_cast<uint8_t*>(launch->workspace) + ctr_off);
  a.status = launch->status;
  a.num_heads = (int)num_heads;
  a.num_kv_heads = (int)Hkv;
  a.num_pages = (int)kv->num_pages;
  a.page_size = (int)kv->page_size;
  a.page_shift = -1;
  for (int sh = 0; sh < 31; ++sh)
    if (kv->page_size == (1u << sh)) a.page_shift = sh;
  a.max_pages = (int)kv->max_pages_per_seq;
  a.split_tiles = (int)split_tiles;
  a.max_splits = (int)max_splits;
  a.scale_log2 = scale * kLog2e;
  a.freq_cis = opts ? opts->freq_cis : nullptr;
  a.rope_positions = opts ? (int)opts->rope_positions : 0;
  a.window = opts ? (int)opts->sliding_window : 0;
  a.softcap = opts ? opts->attn_softcap : 0.0f;
  a.scale = scale;
  a.out_bf16 = (opts && (opts->flags & DOE_DECODE_OUT_BF16)) ? 1 : 0;
  a.inputs_stable = (opts && (opts->flags & DOE_DECODE_INPUTS_STABLE)) ? 1 : 0;
  cudaStream_t st = static_cast<cudaStream_t>(launch->stream);
  // arrival counters of the split stitch start at zero on every launch; the
  // last split of each (sequence, kv head) puts its counter back to zero, so a
  // caller that keeps a workspace for the decode alone may skip the clear
  int rc = DOE_OK;
  if (!(opts && (opts->flags & DOE_DECODE_COUNTERS_ZEROED))) {
    rc = cuda_status(cudaMemsetAsync(a.counters, 0, (size_t)num_seqs * Hkv * sizeof(unsigned), st),
                     "cudaMemsetAsync(split counters)");
    if (rc != DOE_OK) return rc;
  }
  dim3 grid(max_splits, Hkv, num_seqs);
  const bool int8 = kv->kv_dtype == DOE_KV_INT8;
  // K/V pools as {128 elements, Hkv, rows} tensor maps; one box = 16 rows of
  // one kv head: 64 f16 (two boxes per row) or 128 int8.
  for (const void* p : {(const void*)kv->k_pool, (const void*)kv->v_pool, (const void*)kv->k_scale,
                        (const void*)kv->v_scale})
    if (reinterpret_cast<uintptr_t>(p) % 16 != 0) {
      set_op_error("doe_paged_decode: pools and scales must be 16-byte aligned");
      return DOE_INVALID_ARGUMENT;
    }
  const uint64_t pool_rows = (uint64_t)kv->num_pages * kv->page_size;
  CUtensorMap mk, mv;
  const CUtensorMapDataType dt = int8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const uint32_t eb = int8 ? 1 : 2, box_inner = int8 ? 128 : 64;
  rc = encode_rows_map(&mk, kv->k_pool, dt, eb, kD, Hkv, pool_rows, box_inner, 16, "doe_paged_decode");
  if (rc == DOE_OK)
    rc = encode_rows_map(&mv, kv->v_pool, dt, eb, kD, Hkv, pool_rows, box_inner, 16, "doe_paged_decode");
  if (rc != DOE_OK) return rc;
  switch (group) {
    case 1: return int8 ? launch_one<true, 1>(mk, mv, a, grid, st) : launch_one<false, 1>(mk, mv, a, grid, st);
    case 2: return int8 ? launch_one<true, 2>(mk, mv, a, grid, st) : launch_one<false, 2>(mk, mv, a, grid, st);
    case 4: return int8 ? launch_one<true, 4>(mk, mv, a, grid, st) : launch_one<false, 4>(mk, mv, a, grid, st);
    case 8: return int8 ? launch_one<true, 8>(mk, mv, a, grid, st) : launch_one<false, 8>(mk, mv, a, grid, st);
    default:
      set_op_error("doe_paged_decode: heads per kv head must be 1, 2, 4 or 8 (got %u)", group);
      return DOE_UNSUPPORTED;
  }
}

}  // namespace doe

namespace doe {

int launch_combine_natural(const float* part_o, const float* part_ml, float* out, int rows,
                           int fixed_len, int split_tokens, int max_splits, int head_dim,
                           cudaStream_t st) {
  CombineArgs ca;
  ca.part_o = part_o;
  ca.part_ml = part_ml;
  ca.out = out;
  ca.seq_lens = nullptr;
  ca.fixed_len = fixed_len;
  ca.cap = fixed_len;
  ca.split_tokens = split_tokens;
  ca.max_splits = max_splits;
  ca.num_kv_heads = rows;
  ca.group = 1;
  ca.head_dim = head_dim;
  int threads = head_dim >= 256 ? 256 : ((head_dim + 31) / 32) * 32;
  if (threads < max_splits) threads = ((max_splits + 31) / 32) * 32;  // one thread per split
  if (threads > 1024) {
    set_op_error("combine: %d splits exceed one block", max_splits);
    return DOE_UNSUPPORTED;
  }
  combine_splits_kernel<false><<<dim3(rows, 1), threads, 0, st>>>(ca);
  return cuda_status(cudaGetLastError(), "combine_splits_kernel");
}

}  // namespace doe
