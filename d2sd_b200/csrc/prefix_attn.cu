// Kernel (a): shared-prefix (level-1) verify attention on sm_100a.
//
// Replaces flashinfer.single_prefill_with_kv_cache(q_all, k_shared, v_shared,
// causal=False, return_lse=True, sm_scale) at generation/verification.py:145-148
// and model/dflash.py:112-115: every query row (all branches x block tokens x
// the G query heads of a kv head) attends the whole shared prefix of its kv
// head. Output convention (FlashInfer's, include/flashinfer/attention/state.cuh):
// normalised O plus the base-2 log-sum-exp lse = m + log2(sum 2^(s*scale*log2e - m)).
//
// Design (one persistent CTA per SM, plan_layout.h for the work partition):
//   warp 8      producer: Q tile pair once per item (TMA); per 128-key tile,
//               for pages in the tensor core's core-matrix order one bulk copy
//               per page (lanes 0-7) for K and for V, else TMA boxes straight
//               from the paged or contiguous cache (128-byte swizzle). K and V
//               have separate rings and release barriers.
//   warp 9      MMA issuer (one thread): S_i = Q_i K^T (tcgen05.mma, smem x smem
//               -> TMEM, M=128 N=128 K=16 steps) and O_i += P_i V (A operand =
//               P_i in TMEM, B = V in smem, MN-major).
//   warps 0-7   two softmax warpgroups, one per 128-row query tile; thread =
//               row = TMEM lane. Online softmax in the log2 domain with a lazy
//               max (O is rescaled in TMEM only when the running max grows by
//               more than 8, i.e. a factor 256, which keeps p <= 256 in bf16).
//               The first 64 keys of P are released to the MMA warp early.
//   warps 10-11 idle; they complete the third warpgroup, whose registers go
//               to the softmax warpgroups (setmaxnreg).
// TMEM: S0 [0,128) S1 [128,256) O0 [256,256+D) O1 [384,384+D); P_i is written
// as packed bf16 over the first 64 columns of S_i.
// The two tiles ping-pong: while warpgroup 0 turns S0 into P0 the tensor core
// runs Q1 K^T and P1 V, and vice versa. At the end of an item each softmax warp
// normalises its 32 rows of O to bf16 and writes them to the item's partial
// slot through 4 KB of shared memory, so the stores are whole row segments.
#include "common.cuh"
#include "plan_layout.h"

namespace d2sd {
namespace {

using namespace plan;

// 12 warps: two softmax warpgroups (0-7) and a third (8-11) holding the TMA
// producer (8) and the MMA issuer (9); warps 10-11 only complete that
// warpgroup. The launch gives every thread kLaunchRegs registers; the third
// warpgroup then gives most of its share to the softmax warpgroups:
// 256 x kSoftmaxRegs + 128 x kSideRegs <= 384 x kLaunchRegs.
constexpr int kNumThreads = 384;
constexpr int kTmaWarp = 8;
constexpr int kMmaWarp = 9;
constexpr int kLaunchRegs = 168;
constexpr int kSoftmaxRegs = 192;
constexpr int kSideRegs = 112;
static_assert(256 * kSoftmaxRegs + 128 * kSideRegs <= kNumThreads * kLaunchRegs,
              "register split above the launch's registers");
constexpr int kPanelBytes = 128 * 128;  // 128 rows x 128 bytes (64 bf16)
constexpr uint32_t kTmemCols = 512;

template <int D>
struct Cfg {
  static constexpr int kPanels = D / 64;
  static constexpr int kTileBytes = 128 * D * 2;  // a 128-row Q tile or 128-key K/V tile
  // K and V rings are released separately: a K stage as soon as both Q.K^T
  // products that read it are done, a V stage after both P.V products
  static constexpr int kKStages = (D == 128) ? 2 : 4;
  static constexpr int kVStages = (D == 128) ? 2 : 4;
  static constexpr int kSmemQ = 0;
  static constexpr int kSmemK = kSmemQ + 2 * kTileBytes;
  static constexpr int kSmemV = kSmemK + kKStages * kTileBytes;
  // epilogue staging: 4 KB per softmax warp (32 rows x 128 bytes of O)
  static constexpr int kSmemStage = kSmemV + kVStages * kTileBytes;
  static constexpr int kSmemBar = kSmemStage + 8 * 4096;
  // barrier indices
  static constexpr int B_QFULL = 0;
  static constexpr int B_QFREE = 1;
  static constexpr int B_KFULL = 2;
  static constexpr int B_VFULL = B_KFULL + kKStages;
  static constexpr int B_KEMPTY = B_VFULL + kVStages;
  static constexpr int B_VEMPTY = B_KEMPTY + kKStages;
  static constexpr int B_SFULL = B_VEMPTY + kVStages;
  static constexpr int B_PHALF = B_SFULL + 2;  // P of keys 0..63 written
  static constexpr int B_PFULL = B_PHALF + 2;
  static constexpr int B_OFINAL = B_PFULL + 2;
  static constexpr int B_OFREE = B_OFINAL + 2;
  static constexpr int kNumBars = B_OFREE + 2;
  static constexpr int kSmemBytes = kSmemBar + kNumBars * 8 + 16 + 1024;  // + align slack
  static_assert(kSmemBytes <= 227 * 1024, "shared memory of one CTA");
};

struct PrefixParams {
  const int32_t* plan;
  const int32_t* page_table;         // nullptr: contiguous KV
  const int32_t* page_table_offset;  // per request
  void* partial;
  int32_t* status;
  int32_t rows_per_box;  // page_size (paged rows) or 128 (contiguous)
  // UMMA-native pages: the (page, head) block of 16 keys is stored in the
  // tensor core's no-swizzle core-matrix order and fetched with one bulk copy
  const uint8_t* k_pages;
  const uint8_t* v_pages;
  int64_t page_stride_bytes;
  int64_t head_stride_bytes;
  int num_pages;
  int32_t G;
  float scale_log2;
};

__device__ __forceinline__ uint32_t s_col(int i) { return static_cast<uint32_t>(i * 128); }
__device__ __forceinline__ uint32_t o_col(int i) { return static_cast<uint32_t>(256 + i * 128); }

// Warp-uniform bounded wait: every lane polls the barrier itself (one warp-wide
// try_wait per poll), which notices a completed phase sooner than one lane
// polling and broadcasting; the warp goes on only if every lane saw it.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort) {
  const bool ok = mbar_wait(bar, parity, abort);
  return __all_sync(0xffffffffu, ok);
}

// 2^x for a pair of x <= 8 on the FMA pipe, to take part of the exponentials
// off the ex2 pipe (16 lanes per clock per SM on sm_100, half the softmax's
// time). Cody-Waite style reduction: x = j + f with j = round(x) through the
// 1.5 * 2^23 rounding constant and f in [-0.5, 0.5]; 2^f by a cubic whose
// coefficients were fitted here for least maximum relative error on that
// interval (7.5e-5, below the 2^-9 rounding of P to bf16); 2^j is added to the
// exponent field. x is clamped at -126 so that 2^j stays a normal number.
__device__ __forceinline__ void exp2_poly2(uint64_t x2, float& p0, float& p1) {
  float x0, x1;
  f2_unpack(x2, x0, x1);
  const uint64_t xc = f2_pack(fmaxf(x0, -126.f), fmaxf(x1, -126.f));
  const uint64_t t = f2_add(xc, f2_pack(12582912.f, 12582912.f));
  const uint64_t r = f2_add(t, f2_pack(-12582912.f, -12582912.f));
  const uint64_t f = f2_fma(r, f2_pack(-1.f, -1.f), xc);
  uint64_t q = f2_fma(f2_pack(0.05517132208f, 0.05517132208f), f,
                      f2_pack(0.24261054397f, 0.24261054397f));
  q = f2_fma(q, f, f2_pack(0.69326096773f, 0.69326096773f));
  q = f2_fma(q, f, f2_pack(0.99992811680f, 0.99992811680f));
  float q0, q1, t0, t1;
  f2_unpack(q, q0, q1);
  f2_unpack(t, t0, t1);
  p0 = __uint_as_float(__float_as_uint(q0) + (__float_as_uint(t0) << 23));
  p1 = __uint_as_float(__float_as_uint(q1) + (__float_as_uint(t1) << 23));
}

// pairs of each 32-key chunk whose exponentials go to exp2_poly2 (bit e = pair
// e): the last pair, one in sixteen. Measured on cfg3 with the truncating pack
// below, kernel (a) per launch: none 119.5 us, pair 15 116 us, pair 0 117 us,
// pair 8 120 us, pairs 7 and 15 120 us, one in thirty-two 116 us; one in four
// or more is slower still (the softmax is bound by instruction issue as much as
// by the ex2 unit), at D 64 as at D 128.
constexpr uint32_t kPolyPairs = 0x8000u;

// P is rounded to bf16 by truncation: one byte permute per pair, where rounding
// to nearest costs two more integer adds on the softmax's critical issue path
// (3% of kernel (a)'s time on cfg3). Truncation drops the bits below bf16's
// 7-bit fraction, on average half a last place: 2^-8 / m of a weight with
// mantissa m in [1, 2); over log-uniform mantissas (softmax weights span many
// octaves) E[1/m] = 1 / (2 ln 2), a mean loss of 0.2818%. The row sum l comes
// from the f32 weights, so that mean loss is divided out of O in the epilogue;
// what remains is zero-mean, between -0.49% and +0.28% of a weight (round to
// nearest: +-0.39%), and averages out over a row's many weights.
constexpr float kTruncBias = 1.0f / (1.0f - 0.002818f);
__device__ __forceinline__ uint32_t pack_bf16x2_trunc(float lo, float hi) {
  return __byte_perm(__float_as_uint(lo), __float_as_uint(hi), 0x7632);
}

// Producer warp. The page indices of a KV tile are fetched by the whole warp
// (lane b reads page b of the tile) one tile ahead of their use, so no copy
// waits on a dependent page-table load. Row-layout caches go through TMA tensor
// boxes issued by lane 0; UMMA-native pages are one bulk copy per page per
// operand, lane b copying page b.
template <int D, bool NATIVE>
__device__ void producer(const CUtensorMap* tm_q, const CUtensorMap* tm_k, const CUtensorMap* tm_v,
                         const PrefixParams& p, uint8_t* smem, uint64_t* bars, volatile int* abort,
                         int item_begin, int item_end) {
  using C = Cfg<D>;
  const int lane = threadIdx.x & 31;
  const int32_t* items = p.plan + p.plan[H_OFF_ITEMS];
  const int G = p.G;
  const int rpb = p.rows_per_box;
  const int boxes = kTileKeys / rpb;  // <= 16
  uint32_t kt = 0;
  bool alive = true;
  for (int it = item_begin; it < item_end && alive; ++it) {
    const int32_t* I = items + it * kItemInts;
    const int r = I[I_REQ], h = I[I_HEAD], t0 = I[I_T0], t1 = I[I_T1];
    const int kv_end = I[I_KV_END], qtok = I[I_QTOK];
    const int base = p.page_table_offset ? p.page_table_offset[r] : 0;
    const int last_page = (kv_end - 1) / rpb;
    // lane b: coordinate of box b of a tile (page index, or first token)
    auto box_coord = [&](int t) -> int {
      const int pos0 = t * kTileKeys + lane * rpb;
      if (p.page_table) {
        int pg = pos0 / rpb;
        if (pg > last_page) pg = last_page;  // finite filler, masked in softmax
        return lane < boxes ? p.page_table[base + pg] : 0;
      }
      return base + pos0;
    };
    int coord = box_coord(t0);
    if (lane == 0) {
      if (it > item_begin && !mbar_wait(&bars[C::B_QFREE], (it - item_begin - 1) & 1, abort))
        alive = false;
      if (alive) {
        mbar_arrive_expect_tx(&bars[C::B_QFULL], 2 * C::kTileBytes);
#pragma unroll
        for (int i = 0; i < 2; ++i) {
#pragma unroll
          for (int pn = 0; pn < C::kPanels; ++pn) {
            tma_load_3d(smem + C::kSmemQ + i * C::kTileBytes + pn * kPanelBytes, tm_q,
                        &bars[C::B_QFULL], pn * 64, h * G, qtok + i * (kTileRows / G));
          }
        }
      }
    }
    alive = __shfl_sync(0xffffffffu, alive ? 1 : 0, 0) != 0;
    for (int t = t0; t < t1 && alive; ++t, ++kt) {
      const int next = (t + 1 < t1) ? box_coord(t + 1) : 0;  // prefetch the next tile's pages
      const int sk = static_cast<int>(kt % C::kKStages);
      const uint32_t uk = kt / C::kKStages;
      const int sv = static_cast<int>(kt % C::kVStages);
      const uint32_t uv = kt / C::kVStages;
      uint8_t* ks = smem + C::kSmemK + sk * C::kTileBytes;
      uint8_t* vs = smem + C::kSmemV + sv * C::kTileBytes;
      for (int kv = 0; kv < 2; ++kv) {
        const int bar_empty = kv ? C::B_VEMPTY + sv : C::B_KEMPTY + sk;
        const uint32_t use = kv ? uv : uk;
        uint64_t* full = &bars[kv ? C::B_VFULL + sv : C::B_KFULL + sk];
        if (lane == 0 && use > 0 && !mbar_wait(&bars[bar_empty], (use - 1) & 1, abort)) alive = false;
        alive = __shfl_sync(0xffffffffu, alive ? 1 : 0, 0) != 0;
        if (!alive) break;
        uint8_t* dst = kv ? vs : ks;
        if (lane == 0) mbar_arrive_expect_tx(full, C::kTileBytes);
        if (NATIVE) {
          constexpr uint32_t kPageBlock = 16 * D * 2;  // one page of one head
          __syncwarp();
          if (lane < boxes) {
            // a page id outside the pool (a corrupt table) reads page 0 or the last page
            const int pg = coord < 0 ? 0 : (coord >= p.num_pages ? p.num_pages - 1 : coord);
            const int64_t off = static_cast<int64_t>(pg) * p.page_stride_bytes +
                                static_cast<int64_t>(h) * p.head_stride_bytes;
            bulk_load(dst + lane * kPageBlock, (kv ? p.v_pages : p.k_pages) + off, kPageBlock, full);
          }
        } else {
          const CUtensorMap* tm = kv ? tm_v : tm_k;
          for (int b = 0; b < boxes; ++b) {
            const int cb = __shfl_sync(0xffffffffu, coord, b);
            const int c1 = p.page_table ? 0 : cb;
            const int c3 = p.page_table ? cb : 0;
            if (lane == 0) {
#pragma unroll
              for (int pn = 0; pn < C::kPanels; ++pn)
                tma_load_4d(dst + pn * kPanelBytes + b * rpb * 128, tm, full, pn * 64, c1, h, c3);
            }
          }
        }
      }
      coord = next;
    }
  }
}

// K in smem: row layout = two 128-byte-swizzled panels of 64 columns; native
// layout = pages of [2 row groups][D/8 chunks][8 rows][16 B] (no swizzle).
// The MMA issuer is one thread whose instruction latencies are all exposed, and
// the tensor core runs ahead of it by little more than one MMA: any work between
// two MMAs of a block idles the tensor pipe. So every descriptor is built once
// and moved with an immediate: the start-address field is the low 14 bits
// (address >> 4) and shared addresses are below 256 KB, so moving a descriptor
// by b bytes adds b >> 4 to its low word without a carry out of the field.
__device__ __forceinline__ uint64_t desc_at(uint64_t d, uint32_t bytes) {
  uint32_t lo, hi;
  asm("mov.b64 {%0, %1}, %2;" : "=r"(lo), "=r"(hi) : "l"(d));
  lo += bytes >> 4;
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "r"(lo), "r"(hi));
  return r;
}

// S_i = Q_i K^T: M=128, N=128 keys, K = D in steps of 16. qd: descriptor of
// Q tile i; kd: descriptor of the K stage. Q and row-layout K are two
// 128-byte-swizzled panels of 64 columns (kPanelBytes apart); native K is pages
// of [2 row groups][D/8 chunks][8 rows][16 B] (16-byte chunks 128 B apart).
template <int D, bool NATIVE>
__device__ __forceinline__ void issue_qk(uint32_t tmem_s, uint64_t qd, uint64_t kd) {
  constexpr uint32_t idesc = umma_idesc_bf16(128, 128, false);
#pragma unroll
  for (int ks = 0; ks < D / 16; ++ks) {
    const uint32_t off = (ks / 4) * kPanelBytes + (ks % 4) * 32;
    umma_ss(tmem_s, desc_at(qd, off), desc_at(kd, NATIVE ? ks * 256 : off), idesc,
            ks > 0 ? 1u : 0u);
  }
}

// O_i (+)= P_i V for the 16-key steps [KS0, KS1): A = P (packed bf16 in the
// first 64 columns of S_i), B = V (MN-major). vd: descriptor of the V stage;
// native V: one page (16 keys = 2 groups of kGroup bytes) per step; row V: 16
// rows of 128 B per step in each 64-column panel.
template <int D, bool NATIVE, int KS0, int KS1>
__device__ __forceinline__ void issue_pv(uint32_t tmem_o, uint32_t tmem_p, uint64_t vd,
                                         bool accumulate) {
  constexpr uint32_t idesc = umma_idesc_bf16(128, D, true);
  constexpr uint32_t kGroup = (D / 8) * 128;
#pragma unroll
  for (int ks = KS0; ks < KS1; ++ks) {
    umma_ts(tmem_o, tmem_p + ks * 8, desc_at(vd, NATIVE ? ks * 2 * kGroup : ks * 16 * 128), idesc,
            (accumulate || ks > 0) ? 1u : 0u);
  }
}

template <int D, bool NATIVE>
__device__ void mma_issuer(const PrefixParams& p, uint8_t* smem, uint64_t* bars, uint32_t tmem,
                           volatile int* abort, int item_begin, int item_end) {
  using C = Cfg<D>;
  constexpr uint32_t kGroup = (D / 8) * 128;
  const int32_t* items = p.plan + p.plan[H_OFF_ITEMS];
  const uint64_t qd0 = umma_desc_sw128(smem_u32(smem + C::kSmemQ), 16, 1024);
  const uint64_t qd1 = desc_at(qd0, C::kTileBytes);
  const uint64_t kd0 = NATIVE ? umma_desc_noswz(smem_u32(smem + C::kSmemK), 128, kGroup)
                              : umma_desc_sw128(smem_u32(smem + C::kSmemK), 16, 1024);
  const uint64_t vd0 = NATIVE ? umma_desc_noswz(smem_u32(smem + C::kSmemV), kGroup, 128)
                              : umma_desc_sw128(smem_u32(smem + C::kSmemV), kPanelBytes, 1024);
  const uint32_t ts0 = tmem + s_col(0), ts1 = tmem + s_col(1);
  const uint32_t to0 = tmem + o_col(0), to1 = tmem + o_col(1);
  uint32_t kt = 0;
  uint32_t pcount[2] = {0, 0};
  for (int it = item_begin; it < item_end; ++it) {
    const int k = it - item_begin;
    const int32_t* I = items + it * kItemInts;
    const int n = I[I_T1] - I[I_T0];
    if (!mbar_wait(&bars[C::B_QFULL], k & 1, abort)) return;
    tc_fence_after();
    {
      const int sk = static_cast<int>(kt % C::kKStages);
      if (!mbar_wait(&bars[C::B_KFULL + sk], (kt / C::kKStages) & 1, abort)) return;
      tc_fence_after();
      const uint64_t kd = desc_at(kd0, sk * C::kTileBytes);
      issue_qk<D, NATIVE>(ts0, qd0, kd);
      umma_commit(&bars[C::B_SFULL + 0]);
      issue_qk<D, NATIVE>(ts1, qd1, kd);
      umma_commit(&bars[C::B_SFULL + 1]);
      umma_commit(&bars[C::B_KEMPTY + sk]);
      if (n == 1) umma_commit(&bars[C::B_QFREE]);
    }
    for (int j = 0; j < n; ++j) {
      const uint32_t cur = kt + j;
      const int sv = static_cast<int>(cur % C::kVStages);
      const bool has_next = j + 1 < n;
      const int skn = static_cast<int>((cur + 1) % C::kKStages);
      const uint64_t vd = desc_at(vd0, sv * C::kTileBytes);
      const uint64_t kdn = desc_at(kd0, skn * C::kTileBytes);
      if (!mbar_wait(&bars[C::B_VFULL + sv], (cur / C::kVStages) & 1, abort)) return;
      // ---- tile 0 ----
      if (j == 0 && k > 0) {
        if (!mbar_wait(&bars[C::B_OFREE + 0], (k - 1) & 1, abort)) return;
      }
      // P.V in two halves: keys 0..63 as soon as their P is in TMEM
      if (!mbar_wait(&bars[C::B_PHALF + 0], pcount[0] & 1, abort)) return;
      tc_fence_after();
      issue_pv<D, NATIVE, 0, 4>(to0, ts0, vd, j > 0);
      if (!mbar_wait(&bars[C::B_PFULL + 0], pcount[0] & 1, abort)) return;
      ++pcount[0];
      tc_fence_after();
      issue_pv<D, NATIVE, 4, 8>(to0, ts0, vd, true);
      if (has_next) {
        if (!mbar_wait(&bars[C::B_KFULL + skn], ((cur + 1) / C::kKStages) & 1, abort)) return;
        tc_fence_after();
        issue_qk<D, NATIVE>(ts0, qd0, kdn);
        umma_commit(&bars[C::B_SFULL + 0]);
      }
      // ---- tile 1 ----
      if (j == 0 && k > 0) {
        if (!mbar_wait(&bars[C::B_OFREE + 1], (k - 1) & 1, abort)) return;
      }
      if (!mbar_wait(&bars[C::B_PHALF + 1], pcount[1] & 1, abort)) return;
      tc_fence_after();
      issue_pv<D, NATIVE, 0, 4>(to1, ts1, vd, j > 0);
      if (!mbar_wait(&bars[C::B_PFULL + 1], pcount[1] & 1, abort)) return;
      ++pcount[1];
      tc_fence_after();
      issue_pv<D, NATIVE, 4, 8>(to1, ts1, vd, true);
      umma_commit(&bars[C::B_VEMPTY + sv]);
      if (has_next) {
        issue_qk<D, NATIVE>(ts1, qd1, kdn);
        umma_commit(&bars[C::B_SFULL + 1]);
        umma_commit(&bars[C::B_KEMPTY + skn]);
        if (j + 2 == n) umma_commit(&bars[C::B_QFREE]);
      }
    }
    umma_commit(&bars[C::B_OFINAL + 0]);
    umma_commit(&bars[C::B_OFINAL + 1]);
    kt += n;
  }
}

template <int D>
__device__ void softmax_role(const PrefixParams& p, uint8_t* smem, uint64_t* bars, uint32_t tmem,
                             volatile int* abort,
                             int item_begin, int item_end) {
  using C = Cfg<D>;
  const int i = threadIdx.x / 128;         // query tile of this warpgroup
  const int wq = (threadIdx.x / 32) & 3;   // warp inside the warpgroup
  const int lane = threadIdx.x & 31;
  const int row = wq * 32 + lane;          // = TMEM lane
  const uint32_t lane_base = tmem + (static_cast<uint32_t>(wq * 32) << 16);
  const int32_t* items = p.plan + p.plan[H_OFF_ITEMS];
  const float sl2 = p.scale_log2;
  uint32_t scount = 0;
  for (int it = item_begin; it < item_end; ++it) {
    const int k = it - item_begin;
    const int32_t* I = items + it * kItemInts;
    const int t0 = I[I_T0], t1 = I[I_T1];
    const int kv_start = I[I_KV_START], kv_end = I[I_KV_END];
    const int slot = (i == 0) ? I[I_SLOT0] : I[I_SLOT1];
    float m_run = -INFINITY, l_run = 0.f;
    for (int t = t0; t < t1; ++t) {
      if (!warp_wait(&bars[C::B_SFULL + i], scount & 1, abort)) return;
      ++scount;
      tc_fence_after();
      uint32_t s[128];
      tmem_ld128_wait(lane_base + s_col(i), s);
      const int pos0 = t * kTileKeys;
      const bool edge = pos0 < kv_start || pos0 + kTileKeys > kv_end;
      if (edge) {  // mask invisible keys
#pragma unroll
        for (int e = 0; e < 128; ++e) {
          const int pos = pos0 + e;
          if (pos < kv_start || pos >= kv_end) s[e] = 0xff800000u;  // -inf
        }
      }
      // row max: 8 independent accumulators, three-input max
      float mx[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) mx[e] = __uint_as_float(s[e]);
#pragma unroll
      for (int e = 8; e < 128; e += 16) {
#pragma unroll
        for (int k = 0; k < 8; ++k)
          mx[k] = fmax3(mx[k], __uint_as_float(s[e + k]), __uint_as_float(s[e + 8 + k]));
      }
      mx[0] = fmax3(mx[0], mx[1], mx[2]);
      mx[3] = fmax3(mx[3], mx[4], mx[5]);
      mx[6] = fmaxf(mx[6], mx[7]);
      mx[0] = fmax3(mx[0], mx[3], mx[6]);
      const float m_tile = mx[0] * sl2;
      // lazy max: keep m_run unless this tile's max exceeds it by more than 8
      // (p <= 2^8 then); when it does, O and l are rescaled by 2^(m_old - m_new)
      // below, after P is written (S registers are free by then)
      float f = 1.f;
      if (t == t0) {
        m_run = m_tile;
      } else if (m_tile > m_run + 8.f) {
        f = fast_exp2(m_run - m_tile);
        m_run = m_tile;
      }
      const float neg_m = -m_run;
      // keys 0..63 of P are released to the MMA warp before the rest is computed,
      // unless a lane of this warp must first rescale O (that happens at the end)
      const bool early = __all_sync(0xffffffffu, f == 1.f);
      auto release_half = [&](int c) {
        if (c == 1 && early) {
          tmem_st_wait();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&bars[C::B_PHALF + i]);
        }
      };
      float sm[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) sm[e] = 0.f;
      if (!edge) {
        // pairs of columns in f32x2 registers: one FMA / one ADD instruction per pair
        const uint64_t sc2 = f2_pack(sl2, sl2), nm2 = f2_pack(neg_m, neg_m);
        uint64_t acc2[4] = {0ull, 0ull, 0ull, 0ull};
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t pk[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const uint64_t x2 = f2_fma(f2_pack(__uint_as_float(s[c * 32 + 2 * e]),
                                               __uint_as_float(s[c * 32 + 2 * e + 1])), sc2, nm2);
            float p0, p1;
            if ((kPolyPairs >> e) & 1u) {
              exp2_poly2(x2, p0, p1);
            } else {
              float x0, x1;
              f2_unpack(x2, x0, x1);
              p0 = fast_exp2(x0);
              p1 = fast_exp2(x1);
            }
            acc2[e & 3] = f2_add(acc2[e & 3], f2_pack(p0, p1));
            pk[e] = pack_bf16x2_trunc(p0, p1);
          }
          tmem_st16(lane_base + s_col(i) + c * 16, pk);
          release_half(c);
        }
        float a0, a1, b0, b1, c0, c1, d0, d1;
        f2_unpack(acc2[0], a0, a1);
        f2_unpack(acc2[1], b0, b1);
        f2_unpack(acc2[2], c0, c1);
        f2_unpack(acc2[3], d0, d1);
        sm[0] = a0; sm[1] = a1; sm[2] = b0; sm[3] = b1; sm[4] = c0; sm[5] = c1; sm[6] = d0; sm[7] = d1;
      } else {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t pk[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const float p0 = fast_exp2(fmaf(__uint_as_float(s[c * 32 + 2 * e]), sl2, neg_m));
            const float p1 = fast_exp2(fmaf(__uint_as_float(s[c * 32 + 2 * e + 1]), sl2, neg_m));
            sm[(2 * e) & 7] += p0;
            sm[(2 * e + 1) & 7] += p1;
            pk[e] = pack_bf16x2_trunc(p0, p1);
          }
          tmem_st16(lane_base + s_col(i) + c * 16, pk);
          release_half(c);
        }
      }
      if (!early) {
        // some lane of this warp rescales O. The TMEM loads and stores are
        // warp-collective (.sync.aligned), so the whole warp runs them, lanes
        // with f = 1 unchanged. O holds the sum up to the previous tile: this
        // tile's S commit follows the previous P.V in issue order, so that P.V
        // has completed
        l_run *= f;
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c) {
          uint32_t o[32];
          tmem_ld32_wait(lane_base + o_col(i) + c * 32, o);
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * f);
          tmem_st32(lane_base + o_col(i) + c * 32, o);
        }
      }
      const float sum = ((sm[0] + sm[1]) + (sm[2] + sm[3])) + ((sm[4] + sm[5]) + (sm[6] + sm[7]));
      l_run += sum;
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (!early) mbar_arrive(&bars[C::B_PHALF + i]);
        mbar_arrive(&bars[C::B_PFULL + i]);
      }
    }
    // ---- epilogue: normalised O and base-2 LSE into the partial slot ----
    if (!warp_wait(&bars[C::B_OFINAL + i], k & 1, abort)) return;
    tc_fence_after();
    if (slot >= 0) {
      // normalised O of this row in bf16 (the precision FlashInfer hands to its
      // merge), base-2 LSE in fp32; the mean truncation loss of P divided out
      const float inv = l_run > 0.f ? kTruncBias / l_run : 0.f;
      uint8_t* sb = reinterpret_cast<uint8_t*>(p.partial) + static_cast<int64_t>(slot) * slot_bytes(D);
      // Each thread holds its own row; storing it directly would scatter every
      // warp store over 32 rows. So each 64-column panel goes through this
      // warp's 4 KB of shared memory (32 rows x 128 B, 16-byte chunk c of row
      // r at chunk c ^ (r & 7): conflict-free both ways) and leaves as four
      // whole 128-byte row segments per store instruction.
      uint8_t* stg = smem + C::kSmemStage + (threadIdx.x / 32) * 4096;
      uint8_t* gw = sb + static_cast<int64_t>(wq * 32) * D * 2;  // this warp's 32 rows
#pragma unroll 1
      for (int pn = 0; pn < D / 64; ++pn) {
#pragma unroll
        for (int hc = 0; hc < 2; ++hc) {
          uint32_t o[32];
          tmem_ld32_wait(lane_base + o_col(i) + pn * 64 + hc * 32, o);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            uint4 v;
            v.x = pack_bf16x2(__uint_as_float(o[8 * e + 0]) * inv, __uint_as_float(o[8 * e + 1]) * inv);
            v.y = pack_bf16x2(__uint_as_float(o[8 * e + 2]) * inv, __uint_as_float(o[8 * e + 3]) * inv);
            v.z = pack_bf16x2(__uint_as_float(o[8 * e + 4]) * inv, __uint_as_float(o[8 * e + 5]) * inv);
            v.w = pack_bf16x2(__uint_as_float(o[8 * e + 6]) * inv, __uint_as_float(o[8 * e + 7]) * inv);
            const int c = hc * 4 + e;
            *reinterpret_cast<uint4*>(stg + lane * 128 + ((c ^ (lane & 7)) << 4)) = v;
          }
        }
        __syncwarp();
#pragma unroll
        for (int k4 = 0; k4 < 8; ++k4) {
          const int r = 4 * k4 + (lane >> 3), c = lane & 7;
          const uint4 v = *reinterpret_cast<const uint4*>(stg + r * 128 + ((c ^ (r & 7)) << 4));
          *reinterpret_cast<uint4*>(gw + static_cast<int64_t>(r) * D * 2 + pn * 128 + c * 16) = v;
        }
        __syncwarp();
      }
      const float lse = l_run > 0.f ? m_run + fast_log2(l_run) : -INFINITY;
      reinterpret_cast<float*>(sb + static_cast<int64_t>(kTileRows) * D * 2)[row] = lse;
    }
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(&bars[C::B_OFREE + i]);
  }
}

template <int D, bool NATIVE>
__global__ void __launch_bounds__(kNumThreads, 1)
    prefix_attention_kernel(const __grid_constant__ CUtensorMap tm_q,
                            const __grid_constant__ CUtensorMap tm_k,
                            const __grid_constant__ CUtensorMap tm_v, const PrefixParams p) {
  using C = Cfg<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kSmemBar);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + C::kNumBars);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
  const int off_cta = p.plan[H_OFF_CTA];
  const int item_begin = p.plan[off_cta + blockIdx.x];
  const int item_end = p.plan[off_cta + blockIdx.x + 1];

  if (threadIdx.x == 0) {
    mbar_init(&bars[C::B_QFULL], 1);
    mbar_init(&bars[C::B_QFREE], 1);
    for (int s = 0; s < C::kKStages; ++s) {
      mbar_init(&bars[C::B_KFULL + s], 1);
      mbar_init(&bars[C::B_KEMPTY + s], 1);
    }
    for (int s = 0; s < C::kVStages; ++s) {
      mbar_init(&bars[C::B_VFULL + s], 1);
      mbar_init(&bars[C::B_VEMPTY + s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars[C::B_SFULL + i], 1);
      mbar_init(&bars[C::B_PHALF + i], 4);
      mbar_init(&bars[C::B_PFULL + i], 4);
      mbar_init(&bars[C::B_OFINAL + i], 1);
      mbar_init(&bars[C::B_OFREE + i], 4);
    }
    *abort = 0;
    fence_mbar_init();
    fence_proxy_async_smem();
  }
  if (warp == kTmaWarp && lane == 0) {
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_v);
  }
  if (warp == kMmaWarp) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // the set-up above overlaps the previous kernel; its outputs (the partial
  // slots it may still read, the cache it may have written) are safe from here
  grid_dep_wait();
  grid_dep_launch();

  if (warp >= 8) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kSideRegs));
    if (warp == kTmaWarp) {
      producer<D, NATIVE>(&tm_q, &tm_k, &tm_v, p, smem, bars, abort, item_begin, item_end);
      __syncwarp();
    } else if (warp == kMmaWarp) {
      if (lane == 0) mma_issuer<D, NATIVE>(p, smem, bars, tmem, abort, item_begin, item_end);
      __syncwarp();
    }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kSoftmaxRegs));
    softmax_role<D>(p, smem, bars, tmem, abort, item_begin, item_end);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
  if (threadIdx.x == 0 && *abort && p.status) atomicExch(p.status, 1);
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
template <int D, bool NATIVE>
int launch(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
           const PrefixParams& prm, int num_ctas, cudaStream_t stream) {
  using C = Cfg<D>;
  static int configured_device = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_device != dev) {
    cudaError_t e = cudaFuncSetAttribute(prefix_attention_kernel<D, NATIVE>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         C::kSmemBytes);
    if (e != cudaSuccess)
      return fail(D2SD_ERR_CUDA, std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e));
    configured_device = dev;
  }
  return launch_pdl(prefix_attention_kernel<D, NATIVE>, dim3(num_ctas), dim3(kNumThreads),
                    C::kSmemBytes, stream, "prefix_attention_kernel", tq, tk, tv, prm);
}

}  // namespace
}  // namespace d2sd

extern "C" int64_t d2sd_partial_slot_bytes(int32_t head_dim) {
  return d2sd::plan::slot_bytes(head_dim);
}

extern "C" int d2sd_prefix_attention(const void* q, int64_t q_stride_token, int64_t q_stride_head,
                                     int64_t num_q_tokens, const void* k, const void* v,
                                     int64_t kv_stride_page, int64_t kv_stride_slot,
                                     int64_t kv_stride_head, int32_t page_size, int32_t kv_format,
                                     int64_t num_pages,
                                     const int32_t* page_table, const int32_t* page_table_offset,
                                     int32_t num_qo_heads, int32_t num_kv_heads, int32_t head_dim,
                                     float sm_scale, const int32_t* plan, int32_t num_ctas,
                                     void* partial, int64_t partial_bytes, int32_t* status,
                                     void* stream) {
  using namespace d2sd;
  if (!q || !k || !v || !plan || !partial || num_q_tokens <= 0 || num_pages <= 0 ||
      num_qo_heads <= 0 || num_kv_heads <= 0 || num_qo_heads % num_kv_heads != 0)
    return fail(D2SD_ERR_INVALID_ARGUMENT, "d2sd_prefix_attention: invalid argument");
  if (num_ctas <= 0) return D2SD_OK;  // empty plan: nothing to attend
  if (head_dim != 64 && head_dim != 128)
    return fail(D2SD_ERR_UNSUPPORTED, "d2sd_prefix_attention: head_dim must be 64 or 128");
  const int G = num_qo_heads / num_kv_heads;
  if (plan::kTileRows % G != 0)
    return fail(D2SD_ERR_UNSUPPORTED, "d2sd_prefix_attention: qo heads per kv head must divide 128");
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(partial) ||
      q_stride_token % 8 || q_stride_head % 8 || kv_stride_slot % 8 || kv_stride_head % 8 ||
      (page_table && kv_stride_page % 8))
    return fail(D2SD_ERR_INVALID_ARGUMENT,
                "d2sd_prefix_attention: pointers must be 16-byte aligned and strides multiples of 8");
  if (page_table && (page_size % 8 != 0 || page_size <= 0 || plan::kTileKeys % page_size != 0))
    return fail(D2SD_ERR_UNSUPPORTED,
                "d2sd_prefix_attention: page_size must be a multiple of 8 dividing 128");
  if (page_table && !page_table_offset)
    return fail(D2SD_ERR_INVALID_ARGUMENT, "d2sd_prefix_attention: page_table_offset is required");
  if (partial_bytes <= 0)
    return fail(D2SD_ERR_WORKSPACE, "d2sd_prefix_attention: empty partial workspace");
  const bool native = kv_format == D2SD_KV_UMMA_PAGES;
  if (kv_format != D2SD_KV_ROWS && !native)
    return fail(D2SD_ERR_INVALID_ARGUMENT, "d2sd_prefix_attention: unknown kv_format");
  if (native && (!page_table || page_size != 16))
    return fail(D2SD_ERR_INVALID_ARGUMENT,
                "d2sd_prefix_attention: UMMA-native pages need a page table and page_size 16");

  CUtensorMap tq, tk, tv;
  {
    const uint64_t dims[3] = {static_cast<uint64_t>(head_dim), static_cast<uint64_t>(num_qo_heads),
                              static_cast<uint64_t>(num_q_tokens)};
    const uint64_t strides[2] = {static_cast<uint64_t>(q_stride_head) * 2,
                                 static_cast<uint64_t>(q_stride_token) * 2};
    const uint32_t box[3] = {64, static_cast<uint32_t>(G), static_cast<uint32_t>(plan::kTileRows / G)};
    int rc = encode_tensor_map(&tq, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, q, 3, dims, strides, box, "q");
    if (rc) return rc;
  }
  int rows_per_box = native ? 16 : 0;
  if (native) {
    tk = tq;  // unused by the native-page kernel
    tv = tq;
  } else {
    uint64_t dims[4], strides[3];
    uint32_t box[4];
    if (page_table) {
      rows_per_box = page_size;
      dims[0] = head_dim;
      dims[1] = page_size;
      dims[2] = num_kv_heads;
      dims[3] = num_pages;
      strides[0] = kv_stride_slot * 2;
      strides[1] = kv_stride_head * 2;
      strides[2] = kv_stride_page * 2;
    } else {
      rows_per_box = 128;
      dims[0] = head_dim;
      dims[1] = num_pages;  // tokens
      dims[2] = num_kv_heads;
      dims[3] = 1;
      strides[0] = kv_stride_slot * 2;
      strides[1] = kv_stride_head * 2;
      strides[2] = static_cast<uint64_t>(kv_stride_slot) * 2 * static_cast<uint64_t>(num_pages);
      if (strides[2] < strides[1]) strides[2] = strides[1] * num_kv_heads;
    }
    box[0] = 64;
    box[1] = static_cast<uint32_t>(rows_per_box);
    box[2] = 1;
    box[3] = 1;
    int rc = encode_tensor_map(&tk, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, k, 4, dims, strides, box, "k");
    if (rc) return rc;
    rc = encode_tensor_map(&tv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, v, 4, dims, strides, box, "v");
    if (rc) return rc;
  }
  PrefixParams prm;
  prm.plan = plan;
  prm.page_table = page_table;
  prm.page_table_offset = page_table_offset;
  prm.partial = partial;
  prm.status = status;
  prm.rows_per_box = rows_per_box;
  prm.k_pages = static_cast<const uint8_t*>(k);
  prm.v_pages = static_cast<const uint8_t*>(v);
  prm.page_stride_bytes = kv_stride_page * 2;
  prm.head_stride_bytes = kv_stride_head * 2;
  prm.num_pages = num_pages;
  prm.G = G;
  prm.scale_log2 = sm_scale * kLog2e;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (native) {
    return head_dim == 128 ? launch<128, true>(tq, tk, tv, prm, num_ctas, st)
                           : launch<64, true>(tq, tk, tv, prm, num_ctas, st);
  }
  return head_dim == 128 ? launch<128, false>(tq, tk, tv, prm, num_ctas, st)
                         : launch<64, false>(tq, tk, tv, prm, num_ctas, st);
}
