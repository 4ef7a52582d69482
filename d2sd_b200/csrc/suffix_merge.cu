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
// One launch covers every branch. Rows are token*G + g (the G query heads of a
// kv head), cut into 128-row tiles; a tile spans tile_blocks whole blocks when
// block_len * G divides 128 (so short blocks fill the tile), else it lies in
// one block. A CTA of 256 threads takes RP rows of one tile (RP = 128 when
// tiles are plenty; 64 .. 8 when few tiles would leave SMs idle, the level 2 of
// the tile then being recomputed by each of its CTAs):
//   phase 1  thread 0 TMA-loads the tile's Q and the keys/values of its blocks
//            and issues S = Q K^T on tcgen05 into TMEM (M=128, N=32 or 64);
//            warps 0-3 (thread = row = TMEM lane) mask (same block, and causal,
//            full or a custom bitmask inside it), exponentiate and write P back
//            to TMEM; thread 0 issues O = P V (A from TMEM, V MN-major). The
//            CTA's rows of O, normalised, are staged in fp32 over the Q/K/V
//            tiles, with their base-2 LSEs.
//   phase 2  (after the previous kernel -- kernel (a) -- has completed) 8-lane
//            groups merge each row's local state with every partial state
//            kernel (a) wrote for its query tile (or a dense prefix state),
//            apply the sink factor and store the row once (with the fused output
//            exchange, into every rank's buffer).
#include "common.cuh"
#include "plan_layout.h"

#include <cstring>

namespace d2sd {
namespace {

using namespace plan;

constexpr int kThreads = 256;
constexpr int kGroups = kThreads / 8;  // 8-lane groups of the merge
constexpr int kMaxBlockLen = 64;
constexpr int kPanelQ = 128 * 128;     // 128 rows x 128 bytes

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
  int32_t rows_per_cta;  // RP: 128, 64, 32, 16 or 8 rows of a 128-row tile
  int32_t tile_blocks;   // blocks one tile spans (its keys: tile_blocks * block_len)
  int32_t num_tokens;    // num_blocks * block_len
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

template <typename T>
struct Fmt;
template <>
struct Fmt<__nv_bfloat16> {
  static constexpr uint32_t kUmma = 1;  // tcgen05 kind::f16 operand format
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
  static constexpr uint32_t kUmma = 0;
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

template <int D, int NK>
struct SCfg {
  static constexpr int kPanels = D / 64;
  static constexpr int kPanelKV = NK * 128;
  static constexpr int kQBytes = 128 * D * 2;
  static constexpr int kKVBytes = NK * D * 2;
  static constexpr int kSmemQ = 0;
  static constexpr int kSmemK = kQBytes;
  static constexpr int kSmemV = kSmemK + kKVBytes;
  // the staged local output [128][D + 4] fp32 reuses (and may extend) the
  // Q/K/V region once both MMAs have completed
  static constexpr int kStageRow = D + 4;
  static constexpr int kStageBytes = kTileRows * kStageRow * 4;
  static constexpr int kRegion =
      kSmemV + kKVBytes > kStageBytes ? kSmemV + kKVBytes : kStageBytes;
  static constexpr int kSmemBar = (kRegion + 63) / 64 * 64;
  static constexpr int kSmemMeta = kSmemBar + 64;
  static constexpr int kSmemBytes = kSmemMeta + kTileRows * 32 + 1024;  // + align slack
};

__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort) {
  int ok = 1;
  if ((threadIdx.x & 31) == 0) ok = mbar_wait(bar, parity, abort) ? 1 : 0;
  ok = __shfl_sync(0xffffffffu, ok, 0);
  if (ok) {
    while (!mbar_try_wait(bar, parity)) {
    }
  }
  return ok != 0;
}

template <typename T, int D, int NK>
__global__ void __launch_bounds__(kThreads, 2)
    suffix_merge_kernel(const __grid_constant__ CUtensorMap tm_q,
                        const __grid_constant__ CUtensorMap tm_k,
                        const __grid_constant__ CUtensorMap tm_v, const SuffixParams p) {
  using C = SCfg<D, NK>;
  constexpr int SP = C::kStageRow;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kSmemBar);  // load, S, O
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 3);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
  RowMeta* meta = reinterpret_cast<RowMeta*>(smem + C::kSmemMeta);
  float* stage = reinterpret_cast<float*>(smem + C::kSmemQ);  // over Q/K/V after the MMAs

  const int gx = blockIdx.x, h = blockIdx.y;
  // 128-row tile rt of token group gx, CTA part `part` = rows [part*RP, part*RP + RP)
  const int RP = p.rows_per_cta;
  const int parts = kTileRows / RP;
  const int rt = blockIdx.z / parts, part = blockIdx.z - (blockIdx.z / parts) * parts;
  const int TB = p.block_len, G = p.G;
  const int KB = p.tile_blocks * TB;  // tokens of the group (its keys)
  const int gt0 = gx * KB;            // first token of the group
  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
  const float sl2 = p.scale_log2;
  // the next kernel may set itself up now; it waits for this one to complete
  grid_dep_launch();

  // ---- row metadata of this CTA's rows from the (static) plan: warps 4-7,
  // idle during the level-2 attention, so the lookups overlap it ----
  if (threadIdx.x >= 128 && threadIdx.x - 128 < RP) {
    const int lr = threadIdx.x - 128;
    const int Rm = rt * kTileRows + part * RP + lr;
    const int tm = Rm / G, gm = Rm - (Rm / G) * G;
    const bool vm = tm < KB && gt0 + tm < p.num_tokens;
    const int tokm = gt0 + tm;
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
    // lse_local is written by the warps that own the row's TMEM lane
    meta[lr].tok = vm ? tokm : -1;
    meta[lr].hq = h * G + gm;
    meta[lr].slot = slot;
    meta[lr].nslots = nslots;
    meta[lr].prow = prow;
  }

  // ---- phase 1: level-2 attention of the tile on tcgen05 (warps 0-3, thread = row) ----
  uint32_t tmem = 0;
  bool ok = true;
  float lse_l = -INFINITY, inv_l = 0.f;
  const int row = threadIdx.x & 127;  // TMEM lane of warps 0-3
  const int tr = (rt * kTileRows + row) / G;  // token of the row inside the group
  if (p.has_local) {
    if (threadIdx.x == 0) {
      for (int b = 0; b < 3; ++b) mbar_init(&bars[b], 1);
      *abort = 0;
      fence_mbar_init();
      fence_proxy_async_smem();
    }
    if (warp == 0) {
      tmem_alloc(tmem_slot, 256);
      tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    tmem = *tmem_slot;
    if (threadIdx.x == 0) {
      mbar_arrive_expect_tx(&bars[0], C::kQBytes + 2 * C::kKVBytes);
#pragma unroll
      for (int pn = 0; pn < C::kPanels; ++pn) {
        if (p.tile_blocks > 1) {  // one box per block of the tile (its T*G rows)
          for (int bi = 0; bi < p.tile_blocks; ++bi)
            tma_load_4d(smem + C::kSmemQ + pn * kPanelQ + bi * TB * G * 128, &tm_q, &bars[0],
                        pn * 64, h * G, 0, gx * p.tile_blocks + bi);
        } else {
          tma_load_4d(smem + C::kSmemQ + pn * kPanelQ, &tm_q, &bars[0], pn * 64, h * G,
                      rt * (kTileRows / G), gx);
        }
        tma_load_3d(smem + C::kSmemK + pn * C::kPanelKV, &tm_k, &bars[0], pn * 64, h, gt0);
        tma_load_3d(smem + C::kSmemV + pn * C::kPanelKV, &tm_v, &bars[0], pn * 64, h, gt0);
      }
      if (mbar_wait(&bars[0], 0, abort)) {
        tc_fence_after();
        constexpr uint32_t idesc = umma_idesc(128, NK, false, Fmt<T>::kUmma);
        const uint32_t a0 = smem_u32(smem + C::kSmemQ);
        const uint32_t b0 = smem_u32(smem + C::kSmemK);
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks) {
          const uint32_t ka = (ks / 4) * kPanelQ + (ks % 4) * 32;
          const uint32_t kb = (ks / 4) * C::kPanelKV + (ks % 4) * 32;
          umma_ss(tmem, umma_desc_sw128(a0 + ka, 16, 1024), umma_desc_sw128(b0 + kb, 16, 1024),
                  idesc, ks > 0 ? 1u : 0u);
        }
        umma_commit(&bars[1]);
      }
    }
    if (warp < 4) {
      const uint32_t lane_base = tmem + (static_cast<uint32_t>(warp * 32) << 16);
      ok = warp_wait(&bars[1], 0, abort);
      if (ok) {
        tc_fence_after();
        uint32_t s[NK];
        tmem_ld32_wait(lane_base, *reinterpret_cast<uint32_t(*)[32]>(&s[0]));
        if (NK == 64)
          tmem_ld32_wait(lane_base + 32, *reinterpret_cast<uint32_t(*)[32]>(&s[32 % NK]));
        // keys of the group are its tokens 0..KB-1: the row sees only its own
        // block's keys, and inside the block the causal / custom / full mask
        uint64_t allowed = 0;
        if (tr < KB && gt0 + tr < p.num_tokens) {
          const int b = tr / TB, pos = tr - (tr / TB) * TB;
          uint64_t w;
          if (p.mask_mode == D2SD_MASK_CAUSAL) w = (pos >= 63) ? ~0ull : ((2ull << pos) - 1ull);
          else if (p.mask_mode == D2SD_MASK_CUSTOM) w = p.custom_mask[gt0 + tr];
          else w = ~0ull;
          if (TB < 64) w &= (1ull << TB) - 1ull;
          allowed = w << (b * TB);  // b * TB < KB <= 64
        }
        float m = -INFINITY;
#pragma unroll
        for (int j = 0; j < NK; ++j) {
          if (!((allowed >> j) & 1ull)) s[j] = 0xff800000u;
          m = fmaxf(m, __uint_as_float(s[j]));
        }
        const float mm = (m == -INFINITY) ? 0.f : m * sl2;
        float l = 0.f;
#pragma unroll
        for (int c = 0; c < NK / 32; ++c) {
          uint32_t pk[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const float p0 = fast_exp2(fmaf(__uint_as_float(s[c * 32 + 2 * e]), sl2, -mm));
            const float p1 = fast_exp2(fmaf(__uint_as_float(s[c * 32 + 2 * e + 1]), sl2, -mm));
            l += p0 + p1;
            pk[e] = Fmt<T>::pack(p0, p1);
          }
          tmem_st16(lane_base + c * 16, pk);
        }
        tmem_st_wait();
        if (l > 0.f) {
          lse_l = mm + fast_log2(l);
          inv_l = 1.f / l;
        }
      }
    }
    tc_fence_before();
    __syncthreads();
    if (threadIdx.x == 0 && !*abort) {
      tc_fence_after();
      constexpr uint32_t idesc = umma_idesc(128, D, true, Fmt<T>::kUmma);
      const uint32_t b0 = smem_u32(smem + C::kSmemV);
#pragma unroll
      for (int ks = 0; ks < NK / 16; ++ks) {
        umma_ts(tmem + 128, tmem + ks * 8, umma_desc_sw128(b0 + ks * 16 * 128, C::kPanelKV, 1024),
                idesc, ks > 0 ? 1u : 0u);
      }
      umma_commit(&bars[2]);
    }
    if (warp < 4) {
      ok = warp_wait(&bars[2], 0, abort) && ok;
      tc_fence_after();
    }
  }

  // ---- phase 1b: this CTA's rows of the local O, normalised, into the fp32
  // stage over the Q/K/V tiles (free once both MMAs completed). Warp w (< 4)
  // owns TMEM lanes [32w, 32w + 32); it takes part if they meet the CTA's rows ----
  if (warp < 4 && warp * 32 < RP * (part + 1) && warp * 32 + 32 > RP * part) {
    const int lr = row - RP * part;
    const bool mine = lr >= 0 && lr < RP;
    if (mine) meta[lr].lse_local = (p.has_local && ok) ? lse_l : -INFINITY;
    if (p.has_local) {
      const uint32_t lane_base = tmem + (static_cast<uint32_t>(warp * 32) << 16);
      const float sc = ok ? inv_l : 0.f;
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c) {
        uint32_t o[32];
        tmem_ld32_wait(lane_base + 128 + c * 32, o);
        if (!mine) continue;
        float4* dst = reinterpret_cast<float4*>(stage + lr * SP + c * 32);
#pragma unroll
        for (int e = 0; e < 8; ++e)
          dst[e] = make_float4(__uint_as_float(o[4 * e]) * sc, __uint_as_float(o[4 * e + 1]) * sc,
                               __uint_as_float(o[4 * e + 2]) * sc, __uint_as_float(o[4 * e + 3]) * sc);
      }
    }
  }
  if (p.has_local) tc_fence_before();
  __syncthreads();
  if (p.has_local && warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
  if (p.has_local && threadIdx.x == 0 && *abort && p.status) atomicExch(p.status, 2);

  // ---- phase 2: merge. The CTA's 32 lane groups of 8 lanes (4 per warp)
  // take its RP rows in passes of 32 rows (GS = 1 group per row), or, with
  // fewer rows, GS = 32 / RP groups per row (in the same warp); a group takes
  // every GS-th slot of its row, 8 lanes across the row's columns (D/8 each),
  // with up to 8 slot rows and all their LSEs in flight before any use; the
  // row's groups then add their partial sums with shuffles.
  // The partial slots come from the previous kernel (kernel (a)): wait for it.
  // Phase 1 read only q and the block's K/V, which precede kernel (a).
  grid_dep_wait();
  constexpr int CPL = D / 8;          // columns per lane
  constexpr int VEC = CPL * 2 / 16;   // 16-byte vectors per lane and slot row
  constexpr int kBatch = 8;           // slot rows in flight per lane
  constexpr int kLseBlocks = 4;       // LSE blocks of 8 slots loaded together
  const int GS = RP >= kGroups ? 1 : kGroups / RP;  // lane groups per row: 1, 2 or 4
  const int passes = RP >= kGroups ? RP / kGroups : 1;
  const int64_t sbytes = slot_bytes(D);
  const uint8_t* part_base = static_cast<const uint8_t*>(p.partial);
  const int gi = warp * 4 + (lane >> 3), j8 = lane & 7;
  const int sg = gi - (gi / GS) * GS;  // slot group of the row
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
#pragma unroll 1
  for (int ps = 0; ps < passes; ++ps) {
    const int lr = GS == 1 ? ps * kGroups + gi : gi / GS;
    const RowMeta mt = meta[lr];
    const bool live = mt.tok >= 0;
    const int nslots = live ? mt.nslots : 0;
    // the group's slots: sg, sg + GS, ...; k-th of them
    const int nmine = nslots > sg ? (nslots - sg + GS - 1) / GS : 0;
    // loops that shuffle run the warp's largest count (rows of a warp may map
    // to different query tiles); lanes past their own count are predicated off
    const int nmine_w = __reduce_max_sync(0xffffffffu, nmine);
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
    // first batch of slot rows and the LSEs of up to 8 * kLseBlocks slots of
    // the group (lane j8 holds the LSE of the group's slot j8 + 8b), all in flight
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
          acc[c * 8 + 2 * k + 1] =
              fmaf(wj, __uint_as_float(u[k] & 0xffff0000u), acc[c * 8 + 2 * k + 1]);
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
        // the row into every rank's output buffer of this epoch's parity, at
        // this rank's head offset (NVLink stores for the peers)
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
  }

  if (p.world > 0) {
    // Arrival. Every CTA publishes its rows (local and NVLink stores) with one
    // GPU-scope acq_rel ticket; the CTA that draws the last ticket has acquired
    // all of them, issues the launch's single system-scope fence and signals
    // every rank once (one NVLink atomic per peer per call), then waits,
    // bounded, until every rank has signalled this rank, so that the kernel
    // completes only when this rank's buffer is whole.
    // The arrival counters alternate with the epoch parity and the waiting CTA
    // resets its own before the kernel completes: a peer can add to the same
    // counter again (epoch + 2) only after this rank has signalled epoch + 1,
    // which its stream does only after this kernel has completed. Hence the
    // count to wait for is world, whatever the grid of this call or the last.
    __syncthreads();
    if (threadIdx.x == 0) {
      unsigned long long* mine = p.peer_ctr[p.rank];
      const unsigned long long ctas =
          static_cast<unsigned long long>(gridDim.x) * gridDim.y * gridDim.z;
      if (atom_add_acq_rel_gpu(mine + X_TICKET, 1ull) == ctas - 1) {
        fence_acq_rel_sys();
        const int par = static_cast<int>(p.epoch & 1);
        for (int d = 0; d < p.world; ++d) red_add_relaxed_sys(p.peer_ctr[d] + X_ARRIVE0 + par, 1ull);
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
// Rows per CTA: a whole 128-row tile when tiles are plenty (two CTAs fit an
// SM), else fewer rows -- more CTAs, and more lane groups per row -- when few
// tiles would leave SMs idle (KV-head sharding over several GPUs leaves each
// rank few heads, and each query tile then has many partial slots to merge).
// RP halves while the doubled CTA count still fits one CTA per SM, and while
// RP is above 32 with fewer CTAs than SMs. Measured on config 3's per-rank
// shapes ((a)+(b) per layer, one-rank exchange): 64 tiles -> RP 32 (256 CTAs;
// 128 CTAs cost 2 us more), 32 tiles -> RP 32 (128 CTAs; 256 cost 1.6 us
// more), 16 tiles -> RP 16, 8 tiles -> RP 8.
int rows_per_cta(int64_t tiles) {
  const int64_t sms = current_sm_count();
  int rp = kTileRows;
  while (rp > 8) {
    const int64_t ctas = tiles * (kTileRows / rp);
    if (ctas * 2 <= sms || (rp > 32 && ctas < sms)) rp /= 2;
    else break;
  }
  return rp;
}

template <typename T, int D, int NK>
int launch_suffix(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                  const SuffixParams& prm, dim3 grid, cudaStream_t stream) {
  using C = SCfg<D, NK>;
  static int configured = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured != dev) {
    cudaError_t e = cudaFuncSetAttribute(suffix_merge_kernel<T, D, NK>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         C::kSmemBytes);
    if (e != cudaSuccess)
      return fail(D2SD_ERR_CUDA, std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e));
    configured = dev;
  }
  return launch_pdl(suffix_merge_kernel<T, D, NK>, grid, dim3(kThreads), C::kSmemBytes, stream,
                    "suffix_merge_kernel", tq, tk, tv, prm);
}

template <typename T>
int dispatch_suffix(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                    const SuffixParams& prm, int D, int NK, dim3 grid, cudaStream_t st) {
  if (D == 128) {
    return NK == 32 ? launch_suffix<T, 128, 32>(tq, tk, tv, prm, grid, st)
                    : launch_suffix<T, 128, 64>(tq, tk, tv, prm, grid, st);
  }
  return NK == 32 ? launch_suffix<T, 64, 32>(tq, tk, tv, prm, grid, st)
                  : launch_suffix<T, 64, 64>(tq, tk, tv, prm, grid, st);
}

struct PeerArgs {
  void* const* out_ptrs = nullptr;
  unsigned long long* const* counters = nullptr;
  int32_t world = 0, rank = 0, head_offset = 0;
  int64_t st = 0, sh = 0, epoch = 0;
};

int suffix_merge_impl(const void* q, int64_t q_stride_token, int64_t q_stride_head,
                      int64_t q_stride_block, const void* k_local, const void* v_local, int64_t kv_stride_token,
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
                  q_stride_token % 8 || q_stride_head % 8 || q_stride_block % 8 ||
                  kv_stride_token % 8 ||
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

  // Tiles: when block_len * G divides 128 (and G >= 2, so that a tile's keys
  // stay within 64), a 128-row tile spans 128 / (block_len * G) whole blocks;
  // otherwise tiles lie inside one block. Without level 2 the blocks do not
  // matter: all tokens of a head form one group.
  const int64_t ntok = static_cast<int64_t>(num_blocks) * block_len;
  if (ntok * G > INT32_MAX / 2)
    return fail(D2SD_ERR_UNSUPPORTED, "d2sd_suffix_merge: too many tokens");
  int64_t tb = block_len, kblk = 1, groups = num_blocks;
  if (!k_local) {
    tb = ntok;
    groups = 1;
  } else if (G >= 2 && tb * G < plan::kTileRows && plan::kTileRows % (tb * G) == 0 &&
             (tb * G) % 8 == 0) {  // each block's rows start on a 1024-byte swizzle period
    kblk = plan::kTileRows / (tb * G);
    groups = (num_blocks + kblk - 1) / kblk;
  }
  const int64_t tiles_per_group = (kblk * tb * G + plan::kTileRows - 1) / plan::kTileRows;
  prm.block_len = static_cast<int32_t>(tb);
  prm.tile_blocks = static_cast<int32_t>(kblk);
  prm.num_tokens = static_cast<int32_t>(ntok);
  const int rp = rows_per_cta(groups * num_kv_heads * tiles_per_group);
  prm.rows_per_cta = rp;
  const dim3 grid(static_cast<unsigned>(groups), static_cast<unsigned>(num_kv_heads),
                  static_cast<unsigned>(tiles_per_group * (plan::kTileRows / rp)));
  const int NK = kblk * tb <= 32 ? 32 : 64;  // keys of a tile (its group's tokens)

  CUtensorMap tq, tk, tv;
  std::memset(&tq, 0, sizeof(tq));
  std::memset(&tk, 0, sizeof(tk));
  std::memset(&tv, 0, sizeof(tv));
  if (k_local) {
    const CUtensorMapDataType tdt =
        dtype == D2SD_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    {
      // q as [blocks, block_len, Hq, D] with its own block stride: token-major
      // tensors and per-block views (a [B, Hq, T, D] tensor transposed to
      // [B, T, Hq, D]) alike are read in place
      const int64_t qsb = q_stride_block ? q_stride_block : block_len * q_stride_token;
      const uint64_t dims[4] = {static_cast<uint64_t>(head_dim),
                                static_cast<uint64_t>(num_qo_heads),
                                static_cast<uint64_t>(block_len), static_cast<uint64_t>(num_blocks)};
      const uint64_t str[3] = {static_cast<uint64_t>(q_stride_head) * 2,
                               static_cast<uint64_t>(q_stride_token) * 2,
                               static_cast<uint64_t>(qsb) * 2};
      const uint32_t box[4] = {64, static_cast<uint32_t>(G),
                               static_cast<uint32_t>(kblk > 1 ? block_len : 128 / G), 1};
      int rc = encode_tensor_map(&tq, tdt, q, 4, dims, str, box, "q");
      if (rc) return rc;
    }
    {
      const uint64_t dims[3] = {static_cast<uint64_t>(head_dim),
                                static_cast<uint64_t>(num_kv_heads), static_cast<uint64_t>(ntok)};
      const uint64_t str[2] = {static_cast<uint64_t>(kv_stride_head) * 2,
                               static_cast<uint64_t>(kv_stride_token) * 2};
      const uint32_t box[3] = {64, 1, static_cast<uint32_t>(NK)};
      int rc = encode_tensor_map(&tk, tdt, k_local, 3, dims, str, box, "k_local");
      if (rc) return rc;
      rc = encode_tensor_map(&tv, tdt, v_local, 3, dims, str, box, "v_local");
      if (rc) return rc;
    }
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == D2SD_DTYPE_BF16)
    return dispatch_suffix<__nv_bfloat16>(tq, tk, tv, prm, head_dim, NK, grid, st);
  return dispatch_suffix<__half>(tq, tk, tv, prm, head_dim, NK, grid, st);
}
}  // namespace
}  // namespace d2sd

extern "C" int d2sd_suffix_merge(const void* q, int64_t q_stride_token, int64_t q_stride_head,
                                 int64_t q_stride_block, const void* k_local, const void* v_local, int64_t kv_stride_token,
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
  return d2sd::suffix_merge_impl(q, q_stride_token, q_stride_head, q_stride_block, k_local,
                                 v_local,
                                 kv_stride_token, kv_stride_head, num_blocks, block_len, mask_mode,
                                 custom_mask, partial, plan, prefix_token, prefix_out,
                                 prefix_out_stride_token, prefix_out_stride_head, prefix_lse,
                                 prefix_lse_stride_token, out, out_stride_token, out_stride_head,
                                 lse, lse_stride_token, sinks, sink_mode, num_qo_heads,
                                 num_kv_heads, head_dim, dtype, sm_scale, status, stream,
                                 d2sd::PeerArgs{});
}

extern "C" int d2sd_suffix_merge_gather(
    const void* q, int64_t q_stride_token, int64_t q_stride_head, int64_t q_stride_block,
    const void* k_local, const void* v_local, int64_t kv_stride_token, int64_t kv_stride_head,
    int32_t num_blocks,
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
  return suffix_merge_impl(q, q_stride_token, q_stride_head, q_stride_block, k_local, v_local,
                           kv_stride_token,
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
