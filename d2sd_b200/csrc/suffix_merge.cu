// Kernel (b): per-block suffix attention fused with the log-sum-exp merge of
// both cascade levels and the GPT-OSS sink rescale, plus the standalone
// merge_state_in_place replacement.
//
// Reference: CascadeGraphRunner._capture/_run_local_merge
// (model/cascade_graph.py:52-60) runs, per branch i, a causal (verify) or full
// (DTA, model/dflash.py:127-133) single_prefill over the branch's own block
// tokens, then merge_state_in_place into the level-1 state; the sink rescale
// out *= sigmoid(lse - sink) follows at generation/verification.py:173-176.
//
// The work is small and memory-bound (the level-2 attention of a block is at
// most 64 keys per row; the merge reads each row's partial states), so this is
// a high-occupancy SIMT kernel: one launch covers every branch; a CTA of 256
// threads takes RP (32, 16 or 8) consecutive rows of one (block, kv head),
// rows being token*G + g for the G query heads of the kv head.
//   phase 1  the block's K/V of the kv head (only the keys the CTA's rows can
//            see) are staged in shared memory; each warp computes the level-2
//            attention of 4 rows, its four 8-lane groups splitting the keys:
//            scores into shared memory, a warp-wide softmax, then P.V with a
//            reduce-scatter that leaves each group one row; the normalised row
//            and its base-2 LSE go to shared memory. Each row's level 2 is
//            computed once.
//   phase 2  (after the previous kernel -- kernel (a) -- has completed) each
//            row's lane groups merge the local state with every partial state
//            kernel (a) wrote for the row's query tile (or with a dense prefix
//            state), apply the sink factor and store the row once; with the
//            fused output exchange the row goes to every rank's buffer.
#include "common.cuh"
#include "plan_layout.h"

#include <cstring>

namespace d2sd {
namespace {

using namespace plan;

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kGroups = kThreads / 8;  // 8-lane groups of the merge
constexpr int kMaxBlockLen = 64;
constexpr int kMaxRows = 32;           // rows of one CTA (4 per warp in phase 1)

struct SuffixParams {
  const void* q;
  int64_t q_st, q_sh;
  const void* k_local;
  const void* v_local;
  int64_t kv_st, kv_sh;
  const int32_t* plan;
  const void* partial;
  const int32_t* prefix_token;
  const void* prefix_out;
  int64_t po_st, po_sh;
  const float* prefix_lse;
  int64_t pl_st;
  void* out;
  int64_t o_st, o_sh;
  float* lse;
  int64_t l_st;
  const float* sinks;
  const uint64_t* custom_mask;
  int32_t* status;
  int32_t has_local;
  int32_t block_len, mask_mode, sink_mode;
  int32_t Hq, G;
  int32_t rows_per_cta;  // RP: 32, 16 or 8
  int32_t rows_per_unit; // rows of one (block, kv head): block_len * G
  float scale_log2;
  // fused output exchange (d2sd_suffix_merge_gather); world == 0: rows go to out
  void* const* peer_out;               // [2][world]: output buffers of each epoch parity
  unsigned long long* const* peer_ctr;  // [world]: each rank's exchange control block
  int32_t world, rank, head_offset;
  int64_t pg_st, pg_sh;
  int64_t epoch;
};

// Exchange control block of one rank (uint64 words, zero before the first call):
// arrivals of the ranks' calls of even / odd epochs, the CTA ticket of the
// running call, and wait statistics of this rank's calls.
constexpr int X_ARRIVE0 = 0;   // + epoch parity
constexpr int X_TICKET = 2;
constexpr int X_WAIT_NS = 3;   // total time the signalling CTA waited for the peers
constexpr int X_WAITS = 4;     // number of completed waits
constexpr int X_WAIT_MAX = 5;  // longest wait

__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

template <typename T>
struct Fmt;
template <>
struct Fmt<__nv_bfloat16> {
  static __device__ __forceinline__ uint32_t pack(float a, float b) { return pack_bf16x2(a, b); }
  // the 8 elements of a 16-byte vector as floats
  static __device__ __forceinline__ void unpack(const uint4& v, float (&f)[8]) {
    const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      f[2 * k] = __uint_as_float(u[k] << 16);
      f[2 * k + 1] = __uint_as_float(u[k] & 0xffff0000u);
    }
  }
};
template <>
struct Fmt<__half> {
  static __device__ __forceinline__ uint32_t pack(float a, float b) {
    __half2 v = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&v);
  }
  static __device__ __forceinline__ void unpack(const uint4& v, float (&f)[8]) {
    const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 x = __half22float2(*reinterpret_cast<const __half2*>(&u[k]));
      f[2 * k] = x.x;
      f[2 * k + 1] = x.y;
    }
  }
};

// Per merge row, written by phase 1, read by phase 2.
struct RowMeta {
  float lse_local;   // base-2 LSE of the level-2 (local) part, -inf if none
  int32_t tok;       // token index, -1 if the row is padding
  int32_t hq;        // query head
  int32_t slot;      // first partial slot of the row's query tile (partial mode)
  int32_t nslots;    // number of partial slots (partial mode)
  int32_t prow;      // row inside the slot
  int32_t pad[2];
};

// Shared memory of a CTA (bytes from a 16-byte aligned base): the block's K
// and V rows [keys][D], the scores / probabilities of phase 1 [warp][key][4
// rows], the normalised local outputs [RP][D + 4] fp32 and the row metadata.
struct SmemLayout {
  int k, v, p, stage, meta, total;
  __host__ __device__ SmemLayout(int keys, int D, int elem) {
    k = 0;
    v = k + keys * D * elem;
    p = v + keys * D * elem;
    stage = p + kWarps * kMaxBlockLen * 16;
    meta = stage + kMaxRows * (D + 4) * 4;
    total = meta + kMaxRows * static_cast<int>(sizeof(RowMeta));
  }
};

__device__ __forceinline__ uint64_t shfl_xor_u64(uint64_t v, int o) {
  return __shfl_xor_sync(0xffffffffu, static_cast<unsigned long long>(v), o);
}

template <typename T, int D>
__global__ void __launch_bounds__(kThreads, 2) suffix_merge_kernel(const SuffixParams p) {
  constexpr int NC = D / 64;  // 64-column chunks of a row
  extern __shared__ __align__(16) uint8_t smem[];
  const int TB = p.block_len, G = p.G, RP = p.rows_per_cta;
  const int blk = blockIdx.x, h = blockIdx.y, r0 = blockIdx.z * RP;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const SmemLayout sl(p.has_local ? TB : 0, D, static_cast<int>(sizeof(T)));
  float4* pbuf = reinterpret_cast<float4*>(smem + sl.p);
  float* stage = reinterpret_cast<float*>(smem + sl.stage);
  RowMeta* meta = reinterpret_cast<RowMeta*>(smem + sl.meta);
  constexpr int SP = D + 4;  // padded fp32 row of the staged local output
  // the next kernel may set itself up now; it waits for this one to complete
  grid_dep_launch();

  // keys the CTA's rows can see: a causal row of token t sees keys 0..t
  const int t_last = min(TB - 1, (r0 + RP - 1) / G);
  const int nkeys =
      !p.has_local ? 0 : (p.mask_mode == D2SD_MASK_CAUSAL ? t_last + 1 : TB);

  // ---- the block's K/V rows of this kv head into shared memory (loads first,
  // then the row metadata while they are in flight, then the stores) ----
  constexpr int VR = D * static_cast<int>(sizeof(T)) / 16;  // 16-byte vectors per row
  constexpr int EV = 16 / static_cast<int>(sizeof(T));      // elements per vector
  const int nvec = nkeys * VR;
  uint4 kvbuf[4];
  int kvdst[4];
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const int i = threadIdx.x + u * kThreads;
    kvdst[u] = -1;
    if (i < 2 * nvec) {
      const int kv = i >= nvec;
      const int ii = kv ? i - nvec : i;
      const int j = ii / VR, c = ii - (ii / VR) * VR;
      const T* src = static_cast<const T*>(kv ? p.v_local : p.k_local) +
                     static_cast<int64_t>(blk * TB + j) * p.kv_st +
                     static_cast<int64_t>(h) * p.kv_sh + c * EV;
      kvbuf[u] = *reinterpret_cast<const uint4*>(src);
      kvdst[u] = (kv ? sl.v : sl.k) + ii * 16;
    }
  }
  if (threadIdx.x < RP) {
    // row metadata from the (static) plan: the partial slots of the row's query tile
    const int lr = threadIdx.x;
    const int Rm = r0 + lr;
    const int tm = Rm / G, gm = Rm - (Rm / G) * G;
    const bool vm = tm < TB;
    const int tokm = blk * TB + tm;
    int slot = 0, nslots = 0, prow = 0;
    if (vm && p.partial) {
      const int32_t* pl = p.plan;
      const int ptok = p.prefix_token ? p.prefix_token[tokm] : tokm;
      const int req = (ptok >= 0 && ptok < pl[H_NUM_TOKENS]) ? pl[pl[H_OFF_TOKENS] + ptok] : -1;
      if (req >= 0) {
        const int32_t* rq = pl + pl[H_OFF_REQUESTS] + req * kReqInts;
        const int qrow = (ptok - rq[2]) * G + gm;
        const int32_t* un =
            pl + pl[H_OFF_UNITS] + (rq[0] + h * rq[1] + qrow / kTileRows) * kUnitInts;
        slot = un[0];
        nslots = un[1];
        prow = qrow % kTileRows;
      }
    }
    meta[lr].lse_local = -INFINITY;
    meta[lr].tok = vm ? tokm : -1;
    meta[lr].hq = h * G + gm;
    meta[lr].slot = slot;
    meta[lr].nslots = nslots;
    meta[lr].prow = prow;
  }
#pragma unroll
  for (int u = 0; u < 4; ++u)
    if (kvdst[u] >= 0) *reinterpret_cast<uint4*>(smem + kvdst[u]) = kvbuf[u];
  for (int i = threadIdx.x + 4 * kThreads; i < 2 * nvec; i += kThreads) {  // block_len > 32 at D 128
    const int kv = i >= nvec;
    const int ii = kv ? i - nvec : i;
    const int j = ii / VR, c = ii - (ii / VR) * VR;
    const T* src = static_cast<const T*>(kv ? p.v_local : p.k_local) +
                   static_cast<int64_t>(blk * TB + j) * p.kv_st + static_cast<int64_t>(h) * p.kv_sh +
                   c * EV;
    *reinterpret_cast<uint4*>(smem + (kv ? sl.v : sl.k) + ii * 16) =
        *reinterpret_cast<const uint4*>(src);
  }
  __syncthreads();

  // ---- phase 1: level-2 attention, 4 rows per warp. Lane j8 of 8-lane group
  // gi holds columns {c*64 + 8*j8 + e}; for the scores and P.V the groups split
  // the keys (group gi takes keys gi, gi+4, ...) ----
  if (p.has_local && warp * 4 < RP) {
    const int gi = lane >> 3, j8 = lane & 7;
    const float sl2 = p.scale_log2;
    uint64_t allowed[4];
    uint64_t qf[4][NC * 4];  // the rows' q at this lane's columns, fp32 pairs
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int R = r0 + 4 * warp + r;
      const int t = R / G, g = R - (R / G) * G;
      const bool valid = t < TB;
      const int tok = blk * TB + t;
      uint64_t m = 0;
      if (valid) {
        if (p.mask_mode == D2SD_MASK_CAUSAL) m = (t >= 63) ? ~0ull : ((2ull << t) - 1ull);
        else if (p.mask_mode == D2SD_MASK_CUSTOM) m = p.custom_mask[tok];
        else m = ~0ull;
        if (TB < 64) m &= (1ull << TB) - 1ull;
      }
      allowed[r] = m;
#pragma unroll
      for (int c = 0; c < NC; ++c) {
        uint4 raw = make_uint4(0u, 0u, 0u, 0u);
        if (valid)
          raw = *reinterpret_cast<const uint4*>(static_cast<const T*>(p.q) +
                                                static_cast<int64_t>(tok) * p.q_st +
                                                static_cast<int64_t>(h * G + g) * p.q_sh +
                                                c * 64 + 8 * j8);
        float f[8];
        Fmt<T>::unpack(raw, f);
#pragma unroll
        for (int k = 0; k < 4; ++k) qf[r][c * 4 + k] = f2_pack(f[2 * k], f[2 * k + 1]);
      }
    }
    float4* pw = pbuf + warp * kMaxBlockLen;  // [key] -> the 4 rows' scores, then probabilities
    const int iters = (nkeys + 3) / 4;
    for (int it = 0; it < iters; ++it) {
      const int j = gi + 4 * it;
      float d[4] = {0.f, 0.f, 0.f, 0.f};
      if (j < nkeys) {
        uint64_t acc[4] = {0ull, 0ull, 0ull, 0ull};
#pragma unroll
        for (int c = 0; c < NC; ++c) {
          const uint4 kk = *reinterpret_cast<const uint4*>(
              smem + sl.k + (static_cast<int>(j) * D + c * 64 + 8 * j8) * static_cast<int>(sizeof(T)));
          float kf[8];
          Fmt<T>::unpack(kk, kf);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint64_t k2 = f2_pack(kf[2 * k], kf[2 * k + 1]);
#pragma unroll
            for (int r = 0; r < 4; ++r) acc[r] = f2_fma(qf[r][c * 4 + k], k2, acc[r]);
          }
        }
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          float x, y;
          f2_unpack(acc[r], x, y);
          d[r] = x + y;
        }
      }
#pragma unroll
      for (int o = 1; o < 8; o <<= 1)
#pragma unroll
        for (int r = 0; r < 4; ++r) d[r] += __shfl_xor_sync(0xffffffffu, d[r], o);
      if (j8 == 0 && j < nkeys) {
        float4 s;
        s.x = ((allowed[0] >> j) & 1ull) ? d[0] * sl2 : -INFINITY;
        s.y = ((allowed[1] >> j) & 1ull) ? d[1] * sl2 : -INFINITY;
        s.z = ((allowed[2] >> j) & 1ull) ? d[2] * sl2 : -INFINITY;
        s.w = ((allowed[3] >> j) & 1ull) ? d[3] * sl2 : -INFINITY;
        pw[j] = s;
      }
    }
    __syncwarp();
    // softmax of the 4 rows over the keys: lane L holds keys L and L + 32
    const float4 ninf = make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
    float4 sa = lane < nkeys ? pw[lane] : ninf;
    float4 sb = lane + 32 < nkeys ? pw[lane + 32] : ninf;
    float m[4] = {fmaxf(sa.x, sb.x), fmaxf(sa.y, sb.y), fmaxf(sa.z, sb.z), fmaxf(sa.w, sb.w)};
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
      for (int r = 0; r < 4; ++r) m[r] = fmaxf(m[r], __shfl_xor_sync(0xffffffffu, m[r], o));
#pragma unroll
    for (int r = 0; r < 4; ++r) m[r] = (m[r] == -INFINITY) ? 0.f : m[r];
    sa = make_float4(fast_exp2(sa.x - m[0]), fast_exp2(sa.y - m[1]), fast_exp2(sa.z - m[2]),
                     fast_exp2(sa.w - m[3]));
    sb = make_float4(fast_exp2(sb.x - m[0]), fast_exp2(sb.y - m[1]), fast_exp2(sb.z - m[2]),
                     fast_exp2(sb.w - m[3]));
    float l[4] = {sa.x + sb.x, sa.y + sb.y, sa.z + sb.z, sa.w + sb.w};
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
      for (int r = 0; r < 4; ++r) l[r] += __shfl_xor_sync(0xffffffffu, l[r], o);
    if (lane < nkeys) pw[lane] = sa;
    if (lane + 32 < nkeys) pw[lane + 32] = sb;
    __syncwarp();
    // this group's row (gi) after the reduce-scatter below
    const float l_g = gi == 0 ? l[0] : gi == 1 ? l[1] : gi == 2 ? l[2] : l[3];
    const float m_g = gi == 0 ? m[0] : gi == 1 ? m[1] : gi == 2 ? m[2] : m[3];
    const float inv_g = l_g > 0.f ? 1.f / l_g : 0.f;
    const int lr_g = 4 * warp + gi;
    // P.V, 64 columns at a time
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      uint64_t o[4][4];
#pragma unroll
      for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int k = 0; k < 4; ++k) o[r][k] = 0ull;
      for (int it = 0; it < iters; ++it) {
        const int j = gi + 4 * it;
        if (j >= nkeys) break;
        const float4 pj = pw[j];
        const uint4 vv = *reinterpret_cast<const uint4*>(
            smem + sl.v + (j * D + c * 64 + 8 * j8) * static_cast<int>(sizeof(T)));
        float vf[8];
        Fmt<T>::unpack(vv, vf);
        const uint64_t p2[4] = {f2_pack(pj.x, pj.x), f2_pack(pj.y, pj.y), f2_pack(pj.z, pj.z),
                                f2_pack(pj.w, pj.w)};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const uint64_t v2 = f2_pack(vf[2 * k], vf[2 * k + 1]);
#pragma unroll
          for (int r = 0; r < 4; ++r) o[r][k] = f2_fma(p2[r], v2, o[r][k]);
        }
      }
      // reduce-scatter over the four groups: group gi ends with row gi
      const bool hi = (gi & 2) != 0, lo = (gi & 1) != 0;
      uint64_t res[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        uint64_t keep0 = hi ? o[2][k] : o[0][k], send0 = hi ? o[0][k] : o[2][k];
        uint64_t keep1 = hi ? o[3][k] : o[1][k], send1 = hi ? o[1][k] : o[3][k];
        keep0 = f2_add(keep0, shfl_xor_u64(send0, 16));
        keep1 = f2_add(keep1, shfl_xor_u64(send1, 16));
        const uint64_t keep = lo ? keep1 : keep0, send = lo ? keep0 : keep1;
        res[k] = f2_add(keep, shfl_xor_u64(send, 8));
      }
      if (lr_g < RP) {
        float* dst = stage + lr_g * SP + c * 64 + 8 * j8;
        float a0, a1, b0, b1, c0, c1, d0, d1;
        f2_unpack(res[0], a0, a1);
        f2_unpack(res[1], b0, b1);
        f2_unpack(res[2], c0, c1);
        f2_unpack(res[3], d0, d1);
        reinterpret_cast<float4*>(dst)[0] = make_float4(a0 * inv_g, a1 * inv_g, b0 * inv_g, b1 * inv_g);
        reinterpret_cast<float4*>(dst)[1] = make_float4(c0 * inv_g, c1 * inv_g, d0 * inv_g, d1 * inv_g);
      }
    }
    if (j8 == 0 && lr_g < RP) meta[lr_g].lse_local = l_g > 0.f ? m_g + fast_log2(l_g) : -INFINITY;
  }
  __syncthreads();

  // ---- phase 2: merge. The CTA's 32 lane groups of 8 lanes (4 per warp) are
  // spread over its RP rows, GS = 32 / RP groups per row (in the same warp); a
  // group takes every GS-th slot of its row, 8 lanes across the row's columns
  // (D/8 each), with up to 8 slot rows and all their LSEs in flight before any
  // use; the row's groups then add their partial sums with shuffles.
  // The partial slots come from the previous kernel (kernel (a)): wait for it.
  // Phase 1 read only q and the block's K/V, which precede kernel (a).
  grid_dep_wait();
  constexpr int CPL = D / 8;          // columns per lane
  constexpr int VEC = CPL * 2 / 16;   // 16-byte vectors per lane and slot row
  constexpr int kBatch = 8;           // slot rows in flight per lane
  constexpr int kLseBlocks = 4;       // LSE blocks of 8 slots loaded together
  const int GS = kGroups / RP;        // lane groups per row: 1, 2 or 4
  const int64_t sbytes = slot_bytes(D);
  const uint8_t* part_base = static_cast<const uint8_t*>(p.partial);
  const int gi = warp * 4 + (lane >> 3), j8 = lane & 7;
  const int lr = gi / GS, sg = gi - (gi / GS) * GS;  // row, slot group of the row
  const RowMeta mt = meta[lr];
  const bool live = mt.tok >= 0;
  const int nslots = live ? mt.nslots : 0;
  // the group's slots: sg, sg + GS, ...; k-th of them
  const int nmine = nslots > sg ? (nslots - sg + GS - 1) / GS : 0;
  // loops that shuffle run the warp's largest count (rows of a warp may map to
  // different query tiles, e.g. with a shared trunk); lanes past their own
  // count are predicated off
  const int nmine_w = __reduce_max_sync(0xffffffffu, nmine);
  auto gmax = [GS](float v) {  // max over the row's lanes
#pragma unroll
    for (int o = 1; o < 8; o <<= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (GS > 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 8));
    if (GS > 2) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 16));
    return v;
  };
  auto gsum8 = [](float v) {  // sum over the group's 8 lanes
#pragma unroll
    for (int o = 1; o < 8; o <<= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
  };
  auto rsum = [GS](float v) {  // sum over the row's groups (same lane in each)
    if (GS > 1) v += __shfl_xor_sync(0xffffffffu, v, 8);
    if (GS > 2) v += __shfl_xor_sync(0xffffffffu, v, 16);
    return v;
  };
  const uint8_t* prow_base =
      part_base ? part_base + static_cast<int64_t>(mt.prow) * D * 2 + j8 * CPL * 2 : nullptr;
  auto slot_of = [&](int k) { return mt.slot + sg + GS * k; };
  auto slot_lse = [&](int k) -> float {
    return *reinterpret_cast<const float*>(part_base + slot_of(k) * sbytes + kTileRows * D * 2 +
                                           mt.prow * 4);
  };
  auto load_batch = [&](int k0, uint4 (&r)[kBatch][VEC]) {
#pragma unroll
    for (int j = 0; j < kBatch; ++j) {
      if (k0 + j < nmine) {
#pragma unroll
        for (int c = 0; c < VEC; ++c)
          r[j][c] = reinterpret_cast<const uint4*>(prow_base + slot_of(k0 + j) * sbytes)[c];
      }
    }
  };
  // first batch of slot rows and the LSEs of up to 8 * kLseBlocks slots of the
  // group (lane j8 holds the LSE of the group's slot j8 + 8b), all in flight
  uint4 v[kBatch][VEC];
  load_batch(0, v);
  float ls[kLseBlocks];
#pragma unroll
  for (int b = 0; b < kLseBlocks; ++b) ls[b] = (8 * b + j8 < nmine) ? slot_lse(8 * b + j8) : -INFINITY;
  // dense prefix state (no partial slots)
  float lse_p = -INFINITY;
  const T* po = nullptr;
  if (live && !p.partial && p.prefix_out) {
    po = static_cast<const T*>(p.prefix_out) + static_cast<int64_t>(mt.tok) * p.po_st +
         static_cast<int64_t>(mt.hq) * p.po_sh + j8 * CPL;
    lse_p = p.prefix_lse[static_cast<int64_t>(mt.tok) * p.pl_st + mt.hq];
  }
  const float lse_local = live ? mt.lse_local : -INFINITY;
  float lmax = -INFINITY;
#pragma unroll
  for (int b = 0; b < kLseBlocks; ++b) lmax = fmaxf(lmax, ls[b]);
  for (int k0 = 8 * kLseBlocks; k0 < nmine_w; k0 += 8)  // very many slots
    lmax = fmaxf(lmax, k0 + j8 < nmine ? slot_lse(k0 + j8) : -INFINITY);
  const float M = fmaxf(fmaxf(lse_local, lse_p), gmax(lmax));
  const float Mz = (M == -INFINITY) ? 0.f : M;
  const float w_l = (lse_local == -INFINITY) ? 0.f : fast_exp2(lse_local - Mz);
  const float w_p = (lse_p == -INFINITY) ? 0.f : fast_exp2(lse_p - Mz);
  float acc[CPL];
#pragma unroll
  for (int e = 0; e < CPL; ++e) acc[e] = 0.f;
  if (sg == 0) {  // the local and dense-prefix states enter once per row
    if (p.has_local && live) {
      const float4* st = reinterpret_cast<const float4*>(stage + lr * SP + j8 * CPL);
#pragma unroll
      for (int e = 0; e < CPL / 4; ++e) {
        const float4 x = st[e];
        acc[4 * e] = w_l * x.x;
        acc[4 * e + 1] = w_l * x.y;
        acc[4 * e + 2] = w_l * x.z;
        acc[4 * e + 3] = w_l * x.w;
      }
    }
    if (po) {
#pragma unroll
      for (int e = 0; e < CPL; ++e) acc[e] = fmaf(w_p, Num<T>::to_f(po[e]), acc[e]);
    }
  }
  auto add_row = [&](float wj, const uint4 (&r)[VEC]) {
#pragma unroll
    for (int c = 0; c < VEC; ++c) {
      const uint32_t u[4] = {r[c].x, r[c].y, r[c].z, r[c].w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        acc[c * 8 + 2 * k] = fmaf(wj, __uint_as_float(u[k] << 16), acc[c * 8 + 2 * k]);
        acc[c * 8 + 2 * k + 1] = fmaf(wj, __uint_as_float(u[k] & 0xffff0000u), acc[c * 8 + 2 * k + 1]);
      }
    }
  };
  float den = 0.f;
  for (int k0 = 0; k0 < nmine_w; k0 += kBatch) {
    if (k0 > 0) load_batch(k0, v);  // later batches: 8 rows in flight again
    const int b = k0 / 8;
    float l = -INFINITY;
    if (b < kLseBlocks) {
#pragma unroll
      for (int q = 0; q < kLseBlocks; ++q)
        if (q == b) l = ls[q];
    } else if (k0 + j8 < nmine) {
      l = slot_lse(k0 + j8);
    }
    const float w = (l == -INFINITY) ? 0.f : fast_exp2(l - Mz);  // weight of slot k0 + j8
    den += gsum8(w);
#pragma unroll
    for (int j = 0; j < kBatch; ++j) {
      const float wj = __shfl_sync(0xffffffffu, w, (lane & ~7) + j);
      if (k0 + j < nmine) add_row(wj, v[j]);
    }
  }
  // the row's groups add up: acc, den over groups (the local/prefix weights once)
#pragma unroll
  for (int e = 0; e < CPL; ++e) acc[e] = rsum(acc[e]);
  den = rsum(den) + w_l + w_p;
  if (live && sg == 0) {
    const float lse_out = den > 0.f ? Mz + fast_log2(den) : -INFINITY;
    float factor = den > 0.f ? 1.f / den : 0.f;
    if (p.sinks && p.sink_mode != D2SD_SINK_NONE) {
      const float x = (p.sink_mode == D2SD_SINK_EXACT ? lse_out * kLn2 : lse_out) - p.sinks[mt.hq];
      factor *= 1.f / (1.f + __expf(-x));
    }
    uint4 o[VEC];
#pragma unroll
    for (int c = 0; c < VEC; ++c) {
      o[c].x = Fmt<T>::pack(acc[c * 8 + 0] * factor, acc[c * 8 + 1] * factor);
      o[c].y = Fmt<T>::pack(acc[c * 8 + 2] * factor, acc[c * 8 + 3] * factor);
      o[c].z = Fmt<T>::pack(acc[c * 8 + 4] * factor, acc[c * 8 + 5] * factor);
      o[c].w = Fmt<T>::pack(acc[c * 8 + 6] * factor, acc[c * 8 + 7] * factor);
    }
    if (p.world == 0) {
      T* orow = static_cast<T*>(p.out) + static_cast<int64_t>(mt.tok) * p.o_st +
                static_cast<int64_t>(mt.hq) * p.o_sh + j8 * CPL;
#pragma unroll
      for (int c = 0; c < VEC; ++c) reinterpret_cast<uint4*>(orow)[c] = o[c];
    } else {
      // the row into every rank's output buffer of this epoch's parity, at this
      // rank's head offset (NVLink stores for the peers)
      const int64_t off = static_cast<int64_t>(mt.tok) * p.pg_st +
                          static_cast<int64_t>(p.head_offset + mt.hq) * p.pg_sh + j8 * CPL;
      void* const* outs = p.peer_out + (p.epoch & 1) * p.world;
      for (int d = 0; d < p.world; ++d) {
        T* orow = static_cast<T*>(outs[d]) + off;
#pragma unroll
        for (int c = 0; c < VEC; ++c) reinterpret_cast<uint4*>(orow)[c] = o[c];
      }
    }
    if (j8 == 0 && p.lse) p.lse[static_cast<int64_t>(mt.tok) * p.l_st + mt.hq] = lse_out;
  }

  if (p.world > 0) {
    // Arrival. Every CTA makes its peer stores visible system-wide and takes a
    // ticket; the CTA that takes the last one signals every rank once (one
    // NVLink atomic per peer per call instead of one per CTA) and then waits,
    // bounded, until every rank has signalled this rank, so that the kernel
    // completes only when this rank's buffer is whole.
    // The arrival counters alternate with the epoch parity and the waiting CTA
    // resets its own before the kernel completes: a peer can add to the same
    // counter again (epoch + 2) only after this rank has signalled epoch + 1,
    // which its stream does only after this kernel has completed. Hence the
    // count to wait for is world, whatever the grid of this call or the last.
    __syncthreads();
    if (threadIdx.x == 0) {
      __threadfence_system();
      unsigned long long* mine = p.peer_ctr[p.rank];
      const unsigned long long ctas =
          static_cast<unsigned long long>(gridDim.x) * gridDim.y * gridDim.z;
      if (atomicAdd(mine + X_TICKET, 1ull) == ctas - 1) {
        __threadfence_system();
        const int par = static_cast<int>(p.epoch & 1);
        for (int d = 0; d < p.world; ++d) atomicAdd_system(p.peer_ctr[d] + X_ARRIVE0 + par, 1ull);
        const uint64_t t0 = global_timer_ns();
        bool ok = true;
        while (ld_acquire_sys(mine + X_ARRIVE0 + par) < static_cast<unsigned long long>(p.world)) {
          if (global_timer_ns() - t0 > kWaitTimeoutNs) {
            ok = false;
            break;
          }
        }
        const unsigned long long waited = global_timer_ns() - t0;
        if (ok) {
          atomicExch(mine + X_ARRIVE0 + par, 0ull);
          atomicAdd(mine + X_WAIT_NS, waited);
          atomicAdd(mine + X_WAITS, 1ull);
          atomicMax(mine + X_WAIT_MAX, waited);
        } else {
          // a peer never arrived: the counter is left as it is (late arrivals may
          // still land) and the caller must treat the exchange as failed
          atomicExch(p.status, 3);
        }
        atomicExch(mine + X_TICKET, 0ull);
        __threadfence_system();
      }
    }
  }
}

// ---------------------------------------------------------------------------
// merge_state_in_place: (v, s) <- merge((v, s), (v_other, s_other)), base-2.
// Reference: flashinfer.merge_state_in_place at model/cascade_graph.py:58-60.
// ---------------------------------------------------------------------------
template <typename T>
__global__ void merge_state_kernel(T* v, int64_t v_st, int64_t v_sh, float* s, int64_t s_st,
                                   const T* vo, int64_t vo_st, int64_t vo_sh, const float* so,
                                   int64_t so_st, int64_t n, int heads, int D) {
  const int64_t row = blockIdx.x * static_cast<int64_t>(blockDim.y) + threadIdx.y;
  if (row >= n * heads) return;
  const int64_t tok = row / heads;
  const int hd = static_cast<int>(row % heads);
  const float sa = s[tok * s_st + hd];
  const float sb = so[tok * so_st + hd];
  const float M = fmaxf(sa, sb);
  float wa, wb;
  if (M == -INFINITY) {
    wa = 0.f;
    wb = 0.f;
  } else {
    wa = fast_exp2(sa - M);
    wb = fast_exp2(sb - M);
  }
  const float den = wa + wb;
  const float inv = den > 0.f ? 1.f / den : 0.f;
  T* vr = v + tok * v_st + hd * v_sh;
  const T* vor = vo + tok * vo_st + hd * vo_sh;
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    vr[d] = Num<T>::from_f((wa * Num<T>::to_f(vr[d]) + wb * Num<T>::to_f(vor[d])) * inv);
  }
  __syncwarp();
  if (threadIdx.x == 0) s[tok * s_st + hd] = den > 0.f ? M + fast_log2(den) : -INFINITY;
}

}  // namespace
}  // namespace d2sd

namespace d2sd {
namespace {
// Rows per CTA (32, 16 or 8): fewer, and more lane groups per row, when few
// rows would leave most SMs idle (KV-head sharding over several GPUs leaves
// each rank few heads, and each query tile then has many partial slots).
int rows_per_cta(int64_t rows) {
  const int64_t target = 2 * static_cast<int64_t>(current_sm_count());
  int rp = kMaxRows;
  while (rp > 8 && (rows + rp - 1) / rp < target) rp /= 2;
  return rp;
}

template <typename T, int D>
int launch_suffix(const SuffixParams& prm, dim3 grid, int smem, cudaStream_t stream) {
  static int configured = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured != dev) {
    cudaError_t e = cudaFuncSetAttribute(suffix_merge_kernel<T, D>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         SmemLayout(kMaxBlockLen, D, sizeof(T)).total);
    if (e != cudaSuccess)
      return fail(D2SD_ERR_CUDA, std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e));
    configured = dev;
  }
  return launch_pdl(suffix_merge_kernel<T, D>, grid, dim3(kThreads), smem, stream,
                    "suffix_merge_kernel", prm);
}

struct PeerArgs {
  void* const* out_ptrs = nullptr;
  unsigned long long* const* counters = nullptr;
  int32_t world = 0, rank = 0, head_offset = 0;
  int64_t st = 0, sh = 0, epoch = 0;
};

int suffix_merge_impl(const void* q, int64_t q_stride_token, int64_t q_stride_head,
                      const void* k_local, const void* v_local, int64_t kv_stride_token,
                      int64_t kv_stride_head, int32_t num_blocks, int32_t block_len,
                      int32_t mask_mode, const uint64_t* custom_mask, const void* partial,
                      const int32_t* plan, const int32_t* prefix_token, const void* prefix_out,
                      int64_t prefix_out_stride_token, int64_t prefix_out_stride_head,
                      const float* prefix_lse, int64_t prefix_lse_stride_token, void* out,
                      int64_t out_stride_token, int64_t out_stride_head, float* lse,
                      int64_t lse_stride_token, const float* sinks, int32_t sink_mode,
                      int32_t num_qo_heads, int32_t num_kv_heads, int32_t head_dim, int32_t dtype,
                      float sm_scale, int32_t* status, void* stream, const PeerArgs& pa) {
  if (!out || num_blocks < 0 || block_len <= 0 || num_qo_heads <= 0 || num_kv_heads <= 0 ||
      num_qo_heads % num_kv_heads != 0)
    return fail(D2SD_ERR_INVALID_ARGUMENT, "d2sd_suffix_merge: invalid argument");
  if (num_blocks == 0) return D2SD_OK;
  const int G = num_qo_heads / num_kv_heads;
  if (plan::kTileRows % G != 0)
    return fail(D2SD_ERR_UNSUPPORTED, "d2sd_suffix_merge: qo heads per kv head must divide 128");
  if ((k_local == nullptr) != (v_local == nullptr))
    return fail(D2SD_ERR_INVALID_ARGUMENT, "d2sd_suffix_merge: k_local and v_local go together");
  if (k_local && !q)
    return fail(D2SD_ERR_INVALID_ARGUMENT, "d2sd_suffix_merge: q is required with k_local");
  if (k_local && block_len > kMaxBlockLen)
    return fail(D2SD_ERR_UNSUPPORTED, "d2sd_suffix_merge: block_len must be <= 64");
  if (mask_mode == D2SD_MASK_CUSTOM && !custom_mask)
    return fail(D2SD_ERR_INVALID_ARGUMENT, "d2sd_suffix_merge: custom mask pointer missing");
  if (mask_mode < D2SD_MASK_NONE || mask_mode > D2SD_MASK_CUSTOM)
    return fail(D2SD_ERR_INVALID_ARGUMENT, "d2sd_suffix_merge: unknown mask mode");
  if (partial && !plan)
    return fail(D2SD_ERR_INVALID_ARGUMENT, "d2sd_suffix_merge: partial state needs the plan");
  if (!partial && prefix_out && !prefix_lse)
    return fail(D2SD_ERR_INVALID_ARGUMENT, "d2sd_suffix_merge: dense prefix needs its lse");
  if (head_dim != 64 && head_dim != 128)
    return fail(D2SD_ERR_UNSUPPORTED, "d2sd_suffix_merge: head_dim must be 64 or 128");
  if (dtype != D2SD_DTYPE_BF16 && dtype != D2SD_DTYPE_F16)
    return fail(D2SD_ERR_UNSUPPORTED, "d2sd_suffix_merge: dtype must be bf16 or f16");
  if ((out_stride_head % 8) || (out_stride_token % 8) || !aligned16(out))
    return fail(D2SD_ERR_INVALID_ARGUMENT, "d2sd_suffix_merge: out rows must be 16-byte aligned");
  if (partial && (reinterpret_cast<uintptr_t>(partial) & 15u))
    return fail(D2SD_ERR_INVALID_ARGUMENT, "d2sd_suffix_merge: partial must be 16-byte aligned");
  if (k_local && (!aligned16(q) || !aligned16(k_local) || !aligned16(v_local) ||
                  q_stride_token % 8 || q_stride_head % 8 || kv_stride_token % 8 ||
                  kv_stride_head % 8))
    return fail(D2SD_ERR_INVALID_ARGUMENT,
                "d2sd_suffix_merge: q/k/v must be 16-byte aligned with strides multiple of 8");

  SuffixParams prm;
  std::memset(&prm, 0, sizeof(prm));
  prm.q = q;
  prm.q_st = q_stride_token;
  prm.q_sh = q_stride_head;
  prm.k_local = k_local;
  prm.v_local = v_local;
  prm.kv_st = kv_stride_token;
  prm.kv_sh = kv_stride_head;
  prm.plan = plan;
  prm.partial = partial;
  prm.prefix_token = prefix_token;
  prm.prefix_out = partial ? nullptr : prefix_out;
  prm.po_st = prefix_out_stride_token;
  prm.po_sh = prefix_out_stride_head;
  prm.prefix_lse = prefix_lse;
  prm.pl_st = prefix_lse_stride_token;
  prm.out = out;
  prm.o_st = out_stride_token;
  prm.o_sh = out_stride_head;
  prm.lse = lse;
  prm.l_st = lse_stride_token;
  prm.sinks = sinks;
  prm.custom_mask = custom_mask;
  prm.status = status;
  prm.has_local = k_local != nullptr;
  prm.mask_mode = mask_mode;
  prm.sink_mode = sink_mode;
  prm.Hq = num_qo_heads;
  prm.G = G;
  prm.scale_log2 = sm_scale * kLog2e;
  prm.peer_out = pa.out_ptrs;
  prm.peer_ctr = pa.counters;
  prm.world = pa.world;
  prm.rank = pa.rank;
  prm.head_offset = pa.head_offset;
  prm.pg_st = pa.st;
  prm.pg_sh = pa.sh;
  prm.epoch = pa.epoch;

  // a unit is one (block, kv head): block_len * G rows; without level 2 the
  // blocks do not matter and all tokens of a head form one unit
  int64_t units_x = num_blocks, tb = block_len;
  if (!k_local) {
    tb = static_cast<int64_t>(num_blocks) * block_len;
    units_x = 1;
  }
  if (tb * G > INT32_MAX / 2)
    return fail(D2SD_ERR_UNSUPPORTED, "d2sd_suffix_merge: too many tokens");
  prm.block_len = static_cast<int32_t>(tb);
  prm.rows_per_unit = static_cast<int32_t>(tb * G);
  const int rp = rows_per_cta(units_x * num_kv_heads * tb * G);
  prm.rows_per_cta = rp;
  const dim3 grid(static_cast<unsigned>(units_x), static_cast<unsigned>(num_kv_heads),
                  static_cast<unsigned>((tb * G + rp - 1) / rp));
  const int esz = 2;  // bf16 or f16
  const int smem = SmemLayout(k_local ? static_cast<int>(tb) : 0, head_dim, esz).total;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == D2SD_DTYPE_BF16)
    return head_dim == 128 ? launch_suffix<__nv_bfloat16, 128>(prm, grid, smem, st)
                           : launch_suffix<__nv_bfloat16, 64>(prm, grid, smem, st);
  return head_dim == 128 ? launch_suffix<__half, 128>(prm, grid, smem, st)
                         : launch_suffix<__half, 64>(prm, grid, smem, st);
}
}  // namespace
}  // namespace d2sd

extern "C" int d2sd_suffix_merge(const void* q, int64_t q_stride_token, int64_t q_stride_head,
                                 const void* k_local, const void* v_local, int64_t kv_stride_token,
                                 int64_t kv_stride_head, int32_t num_blocks, int32_t block_len,
                                 int32_t mask_mode, const uint64_t* custom_mask,
                                 const void* partial, const int32_t* plan,
                                 const int32_t* prefix_token, const void* prefix_out,
                                 int64_t prefix_out_stride_token, int64_t prefix_out_stride_head,
                                 const float* prefix_lse, int64_t prefix_lse_stride_token,
                                 void* out, int64_t out_stride_token, int64_t out_stride_head,
                                 float* lse, int64_t lse_stride_token, const float* sinks,
                                 int32_t sink_mode, int32_t num_qo_heads, int32_t num_kv_heads,
                                 int32_t head_dim, int32_t dtype, float sm_scale,
                                 int32_t* status, void* stream) {
  return d2sd::suffix_merge_impl(q, q_stride_token, q_stride_head, k_local, v_local,
                                 kv_stride_token, kv_stride_head, num_blocks, block_len, mask_mode,
                                 custom_mask, partial, plan, prefix_token, prefix_out,
                                 prefix_out_stride_token, prefix_out_stride_head, prefix_lse,
                                 prefix_lse_stride_token, out, out_stride_token, out_stride_head,
                                 lse, lse_stride_token, sinks, sink_mode, num_qo_heads,
                                 num_kv_heads, head_dim, dtype, sm_scale, status, stream,
                                 d2sd::PeerArgs{});
}

extern "C" int d2sd_suffix_merge_gather(
    const void* q, int64_t q_stride_token, int64_t q_stride_head, const void* k_local,
    const void* v_local, int64_t kv_stride_token, int64_t kv_stride_head, int32_t num_blocks,
    int32_t block_len, int32_t mask_mode, const uint64_t* custom_mask, const void* partial,
    const int32_t* plan, const int32_t* prefix_token, const void* prefix_out,
    int64_t prefix_out_stride_token, int64_t prefix_out_stride_head, const float* prefix_lse,
    int64_t prefix_lse_stride_token, void* out, int64_t out_stride_token, int64_t out_stride_head,
    float* lse, int64_t lse_stride_token, const float* sinks, int32_t sink_mode,
    int32_t num_qo_heads, int32_t num_kv_heads, int32_t head_dim, int32_t dtype, float sm_scale,
    void* const* out_ptrs, uint64_t* const* counters, int32_t world, int32_t rank,
    int32_t head_offset, int64_t peer_stride_token, int64_t peer_stride_head, int64_t epoch,
    int32_t* status, void* stream) {
  using namespace d2sd;
  if (!out_ptrs || !counters || world <= 0 || rank < 0 || rank >= world || head_offset < 0 ||
      epoch <= 0)
    return fail(D2SD_ERR_INVALID_ARGUMENT, "d2sd_suffix_merge_gather: invalid exchange argument");
  if (!status)
    return fail(D2SD_ERR_INVALID_ARGUMENT,
                "d2sd_suffix_merge_gather: a status word is required (it reports a peer that "
                "never arrived)");
  if (peer_stride_token % 8 || peer_stride_head % 8)
    return fail(D2SD_ERR_INVALID_ARGUMENT,
                "d2sd_suffix_merge_gather: output strides must be multiples of 8 elements");
  PeerArgs pa;
  pa.out_ptrs = out_ptrs;
  pa.counters = reinterpret_cast<unsigned long long* const*>(counters);
  pa.world = world;
  pa.rank = rank;
  pa.head_offset = head_offset;
  pa.st = peer_stride_token;
  pa.sh = peer_stride_head;
  pa.epoch = epoch;
  return suffix_merge_impl(q, q_stride_token, q_stride_head, k_local, v_local, kv_stride_token,
                           kv_stride_head, num_blocks, block_len, mask_mode, custom_mask, partial,
                           plan, prefix_token, prefix_out, prefix_out_stride_token,
                           prefix_out_stride_head, prefix_lse, prefix_lse_stride_token, out,
                           out_stride_token, out_stride_head, lse, lse_stride_token, sinks,
                           sink_mode, num_qo_heads, num_kv_heads, head_dim, dtype, sm_scale,
                           status, stream, pa);
}

extern "C" int d2sd_merge_state(void* v, int64_t v_stride_token, int64_t v_stride_head, float* s,
                                int64_t s_stride_token, const void* v_other, int64_t vo_stride_token,
                                int64_t vo_stride_head, const float* s_other,
                                int64_t so_stride_token, int64_t n, int32_t heads,
                                int32_t head_dim, int32_t dtype, void* stream) {
  using namespace d2sd;
  if (!v || !s || !v_other || !s_other || n < 0 || heads <= 0 || head_dim <= 0)
    return fail(D2SD_ERR_INVALID_ARGUMENT, "d2sd_merge_state: invalid argument");
  if (n == 0) return D2SD_OK;
  const dim3 block(32, 4);
  const int64_t rows = n * heads;
  const dim3 grid(static_cast<unsigned>((rows + 3) / 4));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == D2SD_DTYPE_BF16) {
    merge_state_kernel<__nv_bfloat16><<<grid, block, 0, st>>>(
        static_cast<__nv_bfloat16*>(v), v_stride_token, v_stride_head, s, s_stride_token,
        static_cast<const __nv_bfloat16*>(v_other), vo_stride_token, vo_stride_head, s_other,
        so_stride_token, n, heads, head_dim);
  } else if (dtype == D2SD_DTYPE_F16) {
    merge_state_kernel<__half><<<grid, block, 0, st>>>(
        static_cast<__half*>(v), v_stride_token, v_stride_head, s, s_stride_token,
        static_cast<const __half*>(v_other), vo_stride_token, vo_stride_head, s_other,
        so_stride_token, n, heads, head_dim);
  } else if (dtype == D2SD_DTYPE_F32) {
    merge_state_kernel<float><<<grid, block, 0, st>>>(
        static_cast<float*>(v), v_stride_token, v_stride_head, s, s_stride_token,
        static_cast<const float*>(v_other), vo_stride_token, vo_stride_head, s_other,
        so_stride_token, n, heads, head_dim);
  } else {
    return fail(D2SD_ERR_UNSUPPORTED, "d2sd_merge_state: unknown dtype");
  }
  return check_launch("merge_state_kernel");
}
