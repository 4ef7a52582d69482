// Kernel (c): greedy multi-branch acceptance in one launch.
//
// Reference (generation/d3_generator.py:204-225, with sample() of
// model/utils.py:28-32 at temperature 0):
//   valid = ones(B); acc = 0
//   loop: vb = first b with valid[b]; tok = argmax(logits[vb, acc]); acc += 1
//         emit tok; stop if acc == T; valid &= (block_ids[:, acc] == tok);
//         stop if no branch is valid
// The argmax is a pure function of one logits row, so every row's argmax is
// computed up front (that is the whole cost: B*T*V logits read once, coalesced
// 16-byte loads, HBM-bound); the walk then needs, per step, only whether each
// branch's next draft equals the emitted token, which is precomputed per row as
// a bit mask over the branches. The winning branch returned is vb of the last iteration, the branch
// whose logits produced the bonus token and whose K/V the commit appends
// (generation/d3_generator.py:229-230).
// Ties resolve to the first maximal index and NaN counts as maximal (first NaN
// wins), the torch.argmax convention.
//
// Work: the 16-byte vectors of all logits rows, flattened, are split evenly
// over the grid (stream-K: a CTA's range may cross rows); each thread keeps 8
// loads in flight and each CTA records one (max, first index) per row segment.
// The CTA that finishes last (atomic ticket) reduces the segments of every row,
// forms the rows' match masks (all threads) and runs the walks, one thread per
// request (a shared-memory load and a find-first-set per step).
// Modes: one request (d2sd_verify_accept); a batch of requests with their own
// logits, ids and results in one launch (d2sd_verify_accept_batch, batched
// serving); and a vocabulary-sharded launch (d2sd_verify_accept_sharded) in
// which each rank scans its slice of the vocabulary and the last CTA trades the
// rows' bests with the other ranks over NVLink before every rank walks.
#include <mutex>
#include <string>

#include "common.cuh"

namespace d2sd {
namespace {

constexpr int kThreads = 256;
constexpr int kMaxBranches = 64;

// Total order used by the argmax: larger value first, NaN above everything,
// equal values -> smaller index.
__device__ __forceinline__ bool better(float va, int64_t ia, float vb, int64_t ib) {
  const bool na = va != va, nb = vb != vb;
  if (na || nb) {
    if (na && nb) return ia < ib;
    return na;
  }
  if (va != vb) return va > vb;
  return ia < ib;
}

constexpr int kBatch = 8;       // 16-byte loads in flight per thread

// Stream-K partition of the flattened (row, unit) space over the grid: CTA c
// owns units [c*W, (c+1)*W), W = ceil(total / grid); a unit is one 16-byte
// vector (or one element when rows are not 16-byte aligned).
struct Part {
  int64_t upr;    // units per row
  int64_t total;  // rows * upr
  int64_t W;      // units per CTA
};

__host__ __device__ inline Part partition(int64_t rows, int64_t upr, int64_t grid) {
  Part p;
  p.upr = upr;
  p.total = rows * upr;
  p.W = (p.total + grid - 1) / grid;
  return p;
}

// Segments one row can span: the row's units [r*upr, (r+1)*upr) meet at most
// ceil((upr - 1) / W) + 1 CTA ranges, and upr / W <= grid / rows, so
// ceil(grid / rows) + 2 slots per row always suffice (whatever the vector width).
__host__ __device__ inline int64_t slots_per_row(int64_t rows, int64_t grid) {
  return (grid + rows - 1) / rows + 2;
}

// Per-row records of the scan: CTA c writes the (max, first index) of its part
// of row r into slot c - c_first(r) of the row, and the CTA holding the row's
// last unit writes the row's slot count; the last CTA reads them by row, with
// no division.
struct Workspace {
  unsigned int* ticket;  // CTAs finished; zero between launches
  float* rval;           // [rows][S]
  int64_t* ridx;         // [rows][S]
  int32_t* rcount;       // [rows]
  int64_t S;
};

__host__ __device__ inline int64_t align_up(int64_t x, int64_t a) { return (x + a - 1) / a * a; }

__host__ __device__ inline int64_t workspace_bytes(int64_t rows, int64_t grid) {
  const int64_t n = rows * slots_per_row(rows, grid);
  return 256 + align_up(n * 4, 256) + align_up(n * 8, 256) + align_up(rows * 4, 256);
}

__host__ __device__ inline Workspace carve(void* base, int64_t rows, int64_t grid) {
  uint8_t* b = static_cast<uint8_t*>(base);
  Workspace w;
  w.S = slots_per_row(rows, grid);
  const int64_t n = rows * w.S;
  w.ticket = reinterpret_cast<unsigned int*>(b);
  b += 256;
  w.rval = reinterpret_cast<float*>(b);
  b += align_up(n * 4, 256);
  w.ridx = reinterpret_cast<int64_t*>(b);
  b += align_up(n * 8, 256);
  w.rcount = reinterpret_cast<int32_t*>(b);
  return w;
}

template <typename T>
struct Vec;  // 16-byte vector of T
template <>
struct Vec<float> {
  static constexpr int N = 4;
};
template <>
struct Vec<__nv_bfloat16> {
  static constexpr int N = 8;
};
template <>
struct Vec<__half> {
  static constexpr int N = 8;
};

// NaN-propagating maximum of the elements of one 16-byte vector.
__device__ __forceinline__ float max_nan(float a, float b) {
  float r;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}
template <typename T>
struct VecMax;
template <>
struct VecMax<float> {
  static __device__ __forceinline__ float max(const uint4& v) {
    return max_nan(max_nan(__uint_as_float(v.x), __uint_as_float(v.y)),
                   max_nan(__uint_as_float(v.z), __uint_as_float(v.w)));
  }
  // maximum of a whole batch of vectors (a tree: short dependency chains)
  template <int N>
  static __device__ __forceinline__ float batch(const uint4 (&v)[N]) {
    float m[N];
#pragma unroll
    for (int k = 0; k < N; ++k) m[k] = max(v[k]);
#pragma unroll
    for (int w = 1; w < N; w *= 2)
#pragma unroll
      for (int k = 0; k + w < N; k += 2 * w) m[k] = max_nan(m[k], m[k + w]);
    return m[0];
  }
};
__device__ __forceinline__ uint32_t max_nan_bf16x2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("max.NaN.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t max_nan_f16x2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("max.NaN.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
template <>
struct VecMax<__nv_bfloat16> {
  static __device__ __forceinline__ float max(const uint4& v) {
    const uint32_t m = max_nan_bf16x2(max_nan_bf16x2(v.x, v.y), max_nan_bf16x2(v.z, v.w));
    // bf16 -> f32 is a shift of the bit pattern
    return max_nan(__uint_as_float(m << 16), __uint_as_float(m & 0xffff0000u));
  }
  template <int N>
  static __device__ __forceinline__ float batch(const uint4 (&v)[N]) {
    uint32_t m[N];
#pragma unroll
    for (int k = 0; k < N; ++k)
      m[k] = max_nan_bf16x2(max_nan_bf16x2(v[k].x, v[k].y), max_nan_bf16x2(v[k].z, v[k].w));
#pragma unroll
    for (int w = 1; w < N; w *= 2)
#pragma unroll
      for (int k = 0; k + w < N; k += 2 * w) m[k] = max_nan_bf16x2(m[k], m[k + w]);
    return max_nan(__uint_as_float(m[0] << 16), __uint_as_float(m[0] & 0xffff0000u));
  }
};
template <>
struct VecMax<__half> {
  static __device__ __forceinline__ float max(const uint4& v) {
    const uint32_t m = max_nan_f16x2(max_nan_f16x2(v.x, v.y), max_nan_f16x2(v.z, v.w));
    const __half2 h = *reinterpret_cast<const __half2*>(&m);
    return max_nan(__low2float(h), __high2float(h));
  }
  template <int N>
  static __device__ __forceinline__ float batch(const uint4 (&v)[N]) {
    uint32_t m[N];
#pragma unroll
    for (int k = 0; k < N; ++k)
      m[k] = max_nan_f16x2(max_nan_f16x2(v[k].x, v[k].y), max_nan_f16x2(v[k].z, v[k].w));
#pragma unroll
    for (int w = 1; w < N; w *= 2)
#pragma unroll
      for (int k = 0; k + w < N; k += 2 * w) m[k] = max_nan_f16x2(m[k], m[k + w]);
    const __half2 h = *reinterpret_cast<const __half2*>(&m[0]);
    return max_nan(__low2float(h), __high2float(h));
  }
};

__device__ __forceinline__ void warp_argmax(float& v, int64_t& i) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, o);
    const int64_t oi = __shfl_xor_sync(0xffffffffu, i, o);
    if (better(ov, oi, v, i)) {
      v = ov;
      i = oi;
    }
  }
}

// One thread's scan over units u0, u0+stride, ... < u1 of one row (increasing
// index order). Each 16-byte vector is reduced with a NaN-propagating max;
// only a vector that beats the running best (or holds a NaN) is searched for
// its first maximal index. A strict ">" keeps the first index among equal
// maxima; once the best is NaN nothing replaces it (first NaN wins).
// Whole batches of kBatch vectors take a fast path: the batch's maximum is
// formed from the vectors' maxima (independent of one another, so the chain
// is short), and only a batch whose maximum beats the best -- a handful of
// times per row for any data -- is walked vector by vector with the exact
// rule above. The ragged end of the range goes through the exact rule directly.
template <typename T>
__device__ __forceinline__ void update_vec(const uint4& raw, float vm, int64_t first, float& best_v,
                                           int64_t& best_i) {
  if (!(vm <= best_v) && best_v == best_v) {
    const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
    for (int j = 0; j < Vec<T>::N; ++j) {
      const float x = Num<T>::to_f(e[j]);
      if (x != x || x == vm) {
        best_v = x;
        best_i = first + j;
        break;
      }
    }
  }
}

template <typename T, bool VEC>
__device__ __forceinline__ void scan_units(const T* __restrict__ row, int64_t u0, int64_t u1,
                                           int stride, float& best_v, int64_t& best_i) {
  constexpr int VN = VEC ? Vec<T>::N : 1;
  if (u0 < u1 && best_i == INT64_MAX) best_i = u0 * VN;  // first element seen
  int64_t u = u0;
  if (VEC) {
    const uint4* base = reinterpret_cast<const uint4*>(row);
    const int64_t span = static_cast<int64_t>(stride) * kBatch;
    for (; u + static_cast<int64_t>(stride) * (kBatch - 1) < u1; u += span) {
      const uint4* p = base + u;
      uint4 raw[kBatch];
#pragma unroll
      for (int k = 0; k < kBatch; ++k) raw[k] = __ldg(p + k * stride);
      const float m = VecMax<T>::batch(raw);
      if (!(m <= best_v) && best_v == best_v) {
        // the batch beats the best: its first element equal to m (first NaN
        // if m is NaN) is the new best -- in the first vector whose maximum is m
        int kk = 0;
#pragma unroll
        for (int k = kBatch - 1; k >= 0; --k) {
          const float vk = VecMax<T>::max(raw[k]);
          if (vk == m || (m != m && vk != vk)) kk = k;
        }
        uint4 sel = raw[0];
#pragma unroll
        for (int k = 1; k < kBatch; ++k)
          if (k == kk) sel = raw[k];
        update_vec<T>(sel, m, (u + static_cast<int64_t>(kk) * stride) * VN, best_v, best_i);
      }
    }
    if (u < u1) {  // the ragged end: fewer than kBatch vectors left
      uint4 raw[kBatch];
#pragma unroll
      for (int k = 0; k < kBatch; ++k) {
        const int64_t uu = u + static_cast<int64_t>(k) * stride;
        if (uu < u1) raw[k] = __ldg(base + uu);
      }
#pragma unroll
      for (int k = 0; k < kBatch; ++k) {
        const int64_t uu = u + static_cast<int64_t>(k) * stride;
        if (uu < u1) update_vec<T>(raw[k], VecMax<T>::max(raw[k]), uu * VN, best_v, best_i);
      }
    }
  } else {
    for (; u < u1; u += static_cast<int64_t>(stride) * kBatch) {
#pragma unroll 1
      for (int k = 0; k < kBatch; ++k) {
        const int64_t uu = u + static_cast<int64_t>(k) * stride;
        if (uu >= u1) break;
        const float x = Num<T>::to_f(row[uu]);
        if ((x > best_v || (x != x)) && best_v == best_v) {
          best_v = x;
          best_i = uu;
        }
      }
    }
  }
}

// Logits rows of one launch: num_requests x num_branches x block_len rows,
// row r = (request, branch, position) in that order.
struct Shape {
  int R, B, TB;
  int64_t V;
  int64_t s_r, s_b, s_t;     // logits element strides
  int64_t i_r, i_b, i_t;     // block id strides
  int64_t vocab_offset;      // index of logits column 0 in the full vocabulary
};

// Vocabulary-sharded acceptance: each rank scans its slice of the vocabulary
// and the per-row bests are exchanged over NVLink before the walk.
struct AcceptExchange {
  void* const* rec;                  // [2][world] record buffers ([world][rows] uint4 each)
  unsigned long long* const* ctl;    // [world] control blocks (uint64[8])
  int world, rank;
  int64_t epoch;
  int32_t* status;
};

constexpr int A_ARRIVE0 = 0;  // + epoch parity (control block words)

template <typename T, bool VEC>
__global__ void __launch_bounds__(kThreads, 3)  // the grid is 3 CTAs per SM
    accept_kernel(const T* __restrict__ logits, Shape sh, const int64_t* __restrict__ ids,
                  int32_t* result, int64_t* accepted, int64_t* argmax_out, Workspace ws, Part pt,
                  AcceptExchange ax) {
  __shared__ float sv[kThreads / 32];
  __shared__ int64_t si[kThreads / 32];
  __shared__ bool last;
  // last CTA only (dynamic, rows * 16 bytes): per row its match mask, its
  // argmax and its draft id
  extern __shared__ __align__(16) uint8_t s_dyn[];
  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
  const int TB = sh.TB, B = sh.B;
  const int bt = B * TB;
  const int rows = sh.R * bt;
  // launched with programmatic serialisation: the logits and ids may be
  // written by the previous kernel of the stream
  grid_dep_wait();
  const int64_t u_begin = static_cast<int64_t>(blockIdx.x) * pt.W;
  const int64_t u_end = u_begin + pt.W < pt.total ? u_begin + pt.W : pt.total;
  for (int64_t u = u_begin; u < u_end;) {
    const int64_t r = u / pt.upr;
    const int64_t re = (r + 1) * pt.upr < u_end ? (r + 1) * pt.upr : u_end;
    const int q = static_cast<int>(r / bt);
    const int b = static_cast<int>((r / TB) % B), t = static_cast<int>(r % TB);
    const T* base = logits + static_cast<int64_t>(q) * sh.s_r + static_cast<int64_t>(b) * sh.s_b +
                    static_cast<int64_t>(t) * sh.s_t;
    float bv = -INFINITY;
    int64_t bi = INT64_MAX;
    scan_units<T, VEC>(base, u - r * pt.upr + threadIdx.x, re - r * pt.upr, kThreads, bv, bi);
    warp_argmax(bv, bi);
    if (lane == 0) {
      sv[warp] = bv;
      si[warp] = bi;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      for (int w = 1; w < kThreads / 32; ++w) {
        if (better(sv[w], si[w], bv, bi)) {
          bv = sv[w];
          bi = si[w];
        }
      }
      // this CTA's slot in the row: its index minus that of the row's first CTA
      const int64_t k = blockIdx.x - (r * pt.upr) / pt.W;
      ws.rval[r * ws.S + k] = bv;
      ws.ridx[r * ws.S + k] = bi;
      if (re == (r + 1) * pt.upr) ws.rcount[r] = static_cast<int32_t>(k + 1);  // the row ends here
    }
    __syncthreads();
    u = re;
  }
  // one GPU-scope acq_rel ticket per CTA publishes its segment records; the
  // last CTA's thread 0 acquires them all and the barrier hands them on
  if (threadIdx.x == 0) last = atom_add_acq_rel_gpu(ws.ticket, 1u) == gridDim.x - 1;
  __syncthreads();
  // the next kernel (the commit) may set itself up once every CTA is here; it
  // waits for this whole grid before it reads the results
  grid_dep_launch();
  if (!last) return;

  // ---- last CTA: per-row argmax over the (at most a few) CTA segments of the
  // row and the rows' draft ids into shared memory, then the match masks, then
  // the walks. Each thread keeps the loads of kRowsInFlight rows in flight
  // together (rows do not depend on one another), so the phase costs a couple
  // of round trips to L2 however many rows a thread owns. ----
  uint64_t* s_mask = reinterpret_cast<uint64_t*>(s_dyn);
  int32_t* s_amax = reinterpret_cast<int32_t*>(s_dyn + static_cast<size_t>(rows) * 8);
  int32_t* s_ids = s_amax + rows;
  // (rows that span more than kSlotsInFlight CTAs exist only when rows are
  // fewer than CTAs, i.e. at most one row per thread)
  constexpr int kRowsInFlight = 4, kSlotsInFlight = 2;
  for (int rb = threadIdx.x; rb < rows; rb += kRowsInFlight * kThreads) {
    float v[kRowsInFlight][kSlotsInFlight];
    int64_t ix[kRowsInFlight][kSlotsInFlight];
    int64_t idv[kRowsInFlight];
    int cnt[kRowsInFlight];
#pragma unroll
    for (int j = 0; j < kRowsInFlight; ++j) {
      const int r = rb + j * kThreads;
      if (r < rows) {
        const int q = r / bt, b = (r / TB) % B, t = r % TB;
        idv[j] = __ldg(ids + q * sh.i_r + b * sh.i_b + t * sh.i_t);
        cnt[j] = __ldcg(ws.rcount + r);
        // the first slots of the row, loaded before the count is known (slots
        // past the count hold stale values and are ignored)
#pragma unroll
        for (int k = 0; k < kSlotsInFlight; ++k) {
          if (k < ws.S) {
            v[j][k] = __ldcg(ws.rval + r * ws.S + k);
            ix[j][k] = __ldcg(ws.ridx + r * ws.S + k);
          }
        }
      }
    }
#pragma unroll
    for (int j = 0; j < kRowsInFlight; ++j) {
      const int r = rb + j * kThreads;
      if (r >= rows) break;
      // a draft id no argmax can equal (negative, or beyond 31 bits) becomes -1
      s_ids[r] = (idv[j] >= 0 && idv[j] <= INT32_MAX) ? static_cast<int32_t>(idv[j]) : -1;
      float bv = -INFINITY;
      int64_t bi = INT64_MAX;
#pragma unroll
      for (int k = 0; k < kSlotsInFlight; ++k) {
        if (k < cnt[j] && better(v[j][k], ix[j][k], bv, bi)) {
          bv = v[j][k];
          bi = ix[j][k];
        }
      }
      for (int k = kSlotsInFlight; k < cnt[j]; ++k) {  // rows over more CTAs
        const float vv = __ldcg(ws.rval + r * ws.S + k);
        const int64_t ii = __ldcg(ws.ridx + r * ws.S + k);
        if (better(vv, ii, bv, bi)) {
          bv = vv;
          bi = ii;
        }
      }
      if (bi == INT64_MAX) bi = 0;
      bi += sh.vocab_offset;
      if (ax.world > 0) {
        // the row's best of this vocabulary slice into every rank's buffer
        uint4 rec;
        rec.x = __float_as_uint(bv);
        rec.y = 0u;
        rec.z = static_cast<uint32_t>(static_cast<uint64_t>(bi));
        rec.w = static_cast<uint32_t>(static_cast<uint64_t>(bi) >> 32);
        void* const* outs = ax.rec + (ax.epoch & 1) * ax.world;
        for (int d = 0; d < ax.world; ++d)
          reinterpret_cast<uint4*>(outs[d])[static_cast<int64_t>(ax.rank) * rows + r] = rec;
      } else {
        s_amax[r] = static_cast<int32_t>(bi);
        if (argmax_out) argmax_out[r] = bi;
      }
    }
  }
  if (ax.world > 0) {
    // signal every rank once, wait (bounded) until every rank's records are
    // here, then combine the slices' bests in rank (= vocabulary) order: the
    // first maximal index of the whole row, as the unsharded scan finds it
    __shared__ int s_ok;
    __syncthreads();
    if (threadIdx.x == 0) {
      fence_acq_rel_sys();  // the one system-scope fence of the launch
      const int par = static_cast<int>(ax.epoch & 1);
      for (int d = 0; d < ax.world; ++d) red_add_relaxed_sys(ax.ctl[d] + A_ARRIVE0 + par, 1ull);
      unsigned long long* mine = ax.ctl[ax.rank] + A_ARRIVE0 + par;
      const uint64_t t0 = global_timer_ns();
      int ok = 1;
      while (ld_acquire_sys(mine) < static_cast<unsigned long long>(ax.world)) {
        if (global_timer_ns() - t0 > kWaitTimeoutNs) {
          ok = 0;
          break;
        }
      }
      if (ok) atomicExch(mine, 0ull);
      else atomicExch(ax.status, 3);
      s_ok = ok;
    }
    __syncthreads();  // thread 0's acquire of the peers' records, handed on to the CTA
    const uint4* in = reinterpret_cast<const uint4*>(ax.rec[(ax.epoch & 1) * ax.world + ax.rank]);
    for (int r = threadIdx.x; r < rows; r += kThreads) {
      float bv = -INFINITY;
      int64_t bi = INT64_MAX;
      for (int k = 0; k < ax.world; ++k) {
        const uint4 rec = __ldcv(in + static_cast<int64_t>(k) * rows + r);
        const float vv = __uint_as_float(rec.x);
        const int64_t ii = static_cast<int64_t>((static_cast<uint64_t>(rec.w) << 32) | rec.z);
        if (better(vv, ii, bv, bi)) {
          bv = vv;
          bi = ii;
        }
      }
      if (!s_ok || bi == INT64_MAX) bi = 0;
      s_amax[r] = static_cast<int32_t>(bi);
      if (argmax_out) argmax_out[r] = bi;
    }
  }
  __syncthreads();

  // ---- match masks: row r = (request q, branch b', position t) with argmax
  // tok gets bit b for every branch b whose draft at position t + 1 is tok --
  // the test the walk makes after emitting tok from branch b' at position t ----
  for (int r = threadIdx.x; r < rows; r += kThreads) {
    const int q = r / bt, t = r % TB;
    const int32_t tok = s_amax[r];
    uint64_t m = 0;
    if (t + 1 < TB) {
      const int32_t* id_next = s_ids + q * bt + t + 1;
      for (int b = 0; b < B; ++b) m |= static_cast<uint64_t>(id_next[b * TB] == tok) << b;
    }
    s_mask[r] = m;
  }
  __syncthreads();

  // ---- the acceptance walks, one thread per request: the valid branches as a
  // 64-bit mask, one shared-memory mask per step ----
  for (int q = threadIdx.x; q < sh.R; q += kThreads) {
    const int r0 = q * bt;
    uint64_t valid = (B >= 64) ? ~0ull : ((1ull << B) - 1ull);
    int acc = 0;
    int vb = 0;
    int64_t* acc_q = accepted + static_cast<int64_t>(q) * TB;
    while (true) {
      vb = __ffsll(static_cast<long long>(valid)) - 1;
      const int r = r0 + vb * TB + acc;
      acc_q[acc] = s_amax[r];
      acc += 1;
      if (acc == TB) break;
      valid &= s_mask[r];
      if (valid == 0) break;
    }
    for (int k = acc; k < TB; ++k) acc_q[k] = -1;
    result[2 * q] = acc;
    result[2 * q + 1] = vb;
  }
  if (threadIdx.x == 0) *ws.ticket = 0u;  // leave the workspace zeroed for the next launch
}

}  // namespace
}  // namespace d2sd

namespace d2sd {
namespace {
int accept_grid() { return current_sm_count() * 3; }

template <typename T>
int launch_accept(const void* logits, const Shape& sh, const int64_t* ids, int32_t* result,
                  int64_t* acc_ids, int64_t* argmax_out, void* workspace, int64_t wbytes,
                  const AcceptExchange& ax, cudaStream_t stream, const char* what) {
  constexpr int VN = Vec<T>::N;
  const int64_t rows = static_cast<int64_t>(sh.R) * sh.B * sh.TB;
  const int grid = accept_grid();
  if (rows > 64 * 64)
    return fail(D2SD_ERR_UNSUPPORTED, std::string(what) + ": at most 4096 logits rows");
  if (wbytes < workspace_bytes(rows, grid))
    return fail(D2SD_ERR_WORKSPACE, std::string(what) + ": workspace too small");
  Workspace ws = carve(workspace, rows, grid);
  const bool vec = (reinterpret_cast<uintptr_t>(logits) & 15u) == 0 && sh.V % VN == 0 &&
                   sh.s_r % VN == 0 && sh.s_b % VN == 0 && sh.s_t % VN == 0;
  const int64_t upr = vec ? sh.V / VN : sh.V;
  Part pt = partition(rows, upr, grid);
  // masks, argmaxes and draft ids of the last CTA
  const size_t smem = static_cast<size_t>(rows) * 16;
  // up to 64 KiB of dynamic shared memory (4096 rows) on top of the static part
  // needs the opt-in, once per device and instantiation
  static int configured[2] = {-1, -1};
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured[vec] != dev) {
    cudaError_t e = vec ? cudaFuncSetAttribute(accept_kernel<T, true>,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               64 * 64 * 16)
                        : cudaFuncSetAttribute(accept_kernel<T, false>,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               64 * 64 * 16);
    if (e != cudaSuccess)
      return fail(D2SD_ERR_CUDA, std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e));
    configured[vec] = dev;
  }
  const T* lg = static_cast<const T*>(logits);
  if (vec)
    return launch_pdl(accept_kernel<T, true>, dim3(grid), dim3(kThreads), smem, stream,
                      "accept_kernel", lg, sh, ids, result, acc_ids, argmax_out, ws, pt, ax);
  return launch_pdl(accept_kernel<T, false>, dim3(grid), dim3(kThreads), smem, stream,
                    "accept_kernel", lg, sh, ids, result, acc_ids, argmax_out, ws, pt, ax);
}

int accept_dispatch(const void* logits, int32_t dtype, const Shape& sh, const int64_t* ids,
                    int32_t* result, int64_t* acc_ids, int64_t* argmax_out, void* workspace,
                    int64_t wbytes, const AcceptExchange& ax, void* stream, const char* what) {
  if (!logits || !ids || !result || !acc_ids || !workspace || sh.R <= 0 || sh.B <= 0 ||
      sh.TB <= 0 || sh.V <= 0 || sh.vocab_offset < 0)
    return fail(D2SD_ERR_INVALID_ARGUMENT, std::string(what) + ": invalid argument");
  if (sh.B > kMaxBranches)
    return fail(D2SD_ERR_UNSUPPORTED, std::string(what) + ": at most 64 branches");
  if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0)
    return fail(D2SD_ERR_INVALID_ARGUMENT, std::string(what) + ": workspace must be 256-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case D2SD_DTYPE_F32:
      return launch_accept<float>(logits, sh, ids, result, acc_ids, argmax_out, workspace, wbytes,
                                  ax, st, what);
    case D2SD_DTYPE_BF16:
      return launch_accept<__nv_bfloat16>(logits, sh, ids, result, acc_ids, argmax_out, workspace,
                                          wbytes, ax, st, what);
    case D2SD_DTYPE_F16:
      return launch_accept<__half>(logits, sh, ids, result, acc_ids, argmax_out, workspace,
                                   wbytes, ax, st, what);
    default:
      return fail(D2SD_ERR_UNSUPPORTED, std::string(what) + ": unknown dtype");
  }
}
}  // namespace
}  // namespace d2sd

extern "C" int64_t d2sd_verify_accept_workspace_size(int32_t num_branches, int32_t block_len,
                                                     int64_t vocab) {
  if (num_branches <= 0 || block_len <= 0 || vocab <= 0) return -1;
  return d2sd::workspace_bytes(static_cast<int64_t>(num_branches) * block_len, d2sd::accept_grid());
}

extern "C" int d2sd_verify_accept(const void* logits, int32_t dtype, int32_t num_branches,
                                  int32_t block_len, int64_t vocab, int64_t stride_branch,
                                  int64_t stride_pos, const int64_t* block_ids,
                                  int64_t ids_stride_branch, int64_t ids_stride_pos,
                                  int32_t* result, int64_t* accepted_ids, int64_t* argmax_out,
                                  void* workspace, int64_t workspace_bytes, void* stream) {
  using namespace d2sd;
  const Shape sh{1, num_branches, block_len, vocab, 0, stride_branch, stride_pos,
                 0, ids_stride_branch, ids_stride_pos, 0};
  return accept_dispatch(logits, dtype, sh, block_ids, result, accepted_ids, argmax_out,
                         workspace, workspace_bytes, AcceptExchange{}, stream,
                         "d2sd_verify_accept");
}

extern "C" int64_t d2sd_verify_accept_batch_workspace_size(int32_t num_requests,
                                                           int32_t num_branches,
                                                           int32_t block_len, int64_t vocab) {
  if (num_requests <= 0 || num_branches <= 0 || block_len <= 0 || vocab <= 0) return -1;
  return d2sd::workspace_bytes(static_cast<int64_t>(num_requests) * num_branches * block_len,
                               d2sd::accept_grid());
}

extern "C" int d2sd_verify_accept_batch(const void* logits, int32_t dtype, int32_t num_requests,
                                        int32_t num_branches, int32_t block_len, int64_t vocab,
                                        int64_t stride_request, int64_t stride_branch,
                                        int64_t stride_pos, const int64_t* block_ids,
                                        int64_t ids_stride_request, int64_t ids_stride_branch,
                                        int64_t ids_stride_pos, int32_t* result,
                                        int64_t* accepted_ids, int64_t* argmax_out,
                                        void* workspace, int64_t workspace_bytes, void* stream) {
  using namespace d2sd;
  const Shape sh{num_requests, num_branches, block_len, vocab, stride_request, stride_branch,
                 stride_pos, ids_stride_request, ids_stride_branch, ids_stride_pos, 0};
  return accept_dispatch(logits, dtype, sh, block_ids, result, accepted_ids, argmax_out,
                         workspace, workspace_bytes, AcceptExchange{}, stream,
                         "d2sd_verify_accept_batch");
}

extern "C" int d2sd_verify_accept_sharded(
    const void* logits, int32_t dtype, int32_t num_requests, int32_t num_branches,
    int32_t block_len, int64_t vocab_slice, int64_t vocab_offset, int64_t stride_request,
    int64_t stride_branch, int64_t stride_pos, const int64_t* block_ids,
    int64_t ids_stride_request, int64_t ids_stride_branch, int64_t ids_stride_pos,
    int32_t* result, int64_t* accepted_ids, int64_t* argmax_out, void* workspace,
    int64_t workspace_bytes, void* const* record_ptrs, uint64_t* const* control_ptrs,
    int32_t world, int32_t rank, int64_t epoch, int32_t* status, void* stream) {
  using namespace d2sd;
  if (!record_ptrs || !control_ptrs || !status || world <= 0 || rank < 0 || rank >= world ||
      epoch <= 0)
    return fail(D2SD_ERR_INVALID_ARGUMENT, "d2sd_verify_accept_sharded: invalid exchange argument");
  const Shape sh{num_requests, num_branches, block_len, vocab_slice, stride_request,
                 stride_branch, stride_pos, ids_stride_request, ids_stride_branch,
                 ids_stride_pos, vocab_offset};
  AcceptExchange ax;
  ax.rec = record_ptrs;
  ax.ctl = reinterpret_cast<unsigned long long* const*>(control_ptrs);
  ax.world = world;
  ax.rank = rank;
  ax.epoch = epoch;
  ax.status = status;
  return accept_dispatch(logits, dtype, sh, block_ids, result, accepted_ids, argmax_out,
                         workspace, workspace_bytes, ax, stream, "d2sd_verify_accept_sharded");
}

// ---------------------------------------------------------------------------
// Allocation-free variant of d2sd_verify_accept.
//
// Some callers cannot hand this library a workspace or let it allocate one: a
// serving runtime whose memory planner owns every device allocation up front
// (so that peak memory is known and nothing fragments mid-run), or code that
// runs while a stream is being captured into a CUDA graph, where a cudaMalloc
// is not allowed. For them the acceptance scratch (the per-CTA argmax records
// and the completion ticket) lives in the file-scope array below, 256 KiB,
// which every GPU that loads this library holds until the process exits.
// Requests whose scratch would not fit are rejected with an error.
//
// In host code `g_accept_scratch` is only a host-side stand-in for the device
// array; its device address is fetched with cudaGetSymbolAddress, once per
// device, on the first call made with that device current (and again if the
// device's context has changed since, as after cudaDeviceReset). That first
// call should therefore happen before any stream capture. All calls share the one
// array and it keeps the previous call's contents: the ticket is cleared on
// the caller's stream before every launch, and calls whose kernels overlap on
// the GPU (e.g. issued on two streams at once) race on the array.
// ---------------------------------------------------------------------------
namespace d2sd {
namespace {

constexpr int64_t kStaticScratchBytes = 256 * 1024;
static __device__ __align__(256) uint8_t g_accept_scratch[kStaticScratchBytes];

// Unique id of the current CUDA context (cuCtxGetId through the runtime's
// driver entry point), 0 if it cannot be read. A device reset or a recreated
// primary context gets a new id, and with it a new copy of the array.
unsigned long long current_context_id() {
  using GetCur = CUresult (*)(CUcontext*);
  using GetId = CUresult (*)(CUcontext, unsigned long long*);
  static GetCur get_cur = nullptr;
  static GetId get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &p, 4000, cudaEnableDefault, &q) ==
            cudaSuccess && q == cudaDriverEntryPointSuccess)
      get_cur = reinterpret_cast<GetCur>(p);
    if (cudaGetDriverEntryPointByVersion("cuCtxGetId", &p, 12000, cudaEnableDefault, &q) ==
            cudaSuccess && q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<GetId>(p);
  });
  CUcontext ctx = nullptr;
  unsigned long long id = 0;
  if (!get_cur || !get_id || get_cur(&ctx) != CUDA_SUCCESS || ctx == nullptr ||
      get_id(ctx, &id) != CUDA_SUCCESS)
    return 0;
  return id;
}

int static_scratch(void** out) {
  static std::mutex mu;
  static void* addr[64] = {};
  static unsigned long long ctx_of[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess)
    return fail(D2SD_ERR_CUDA, std::string("cudaGetDevice: ") + cudaGetErrorString(e));
  if (dev < 0 || dev >= 64)
    return fail(D2SD_ERR_UNSUPPORTED, "d2sd_verify_accept_noalloc: device index above 63");
  std::lock_guard<std::mutex> lock(mu);
  const unsigned long long ctx = current_context_id();
  // the address is looked up again whenever the context changed (or its id is
  // unknown), so it never outlives a device reset
  if (addr[dev] == nullptr || ctx == 0 || ctx != ctx_of[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_accept_scratch);
    if (e != cudaSuccess || p == nullptr)
      return fail(D2SD_ERR_CUDA, std::string("cudaGetSymbolAddress(g_accept_scratch): ") +
                                     cudaGetErrorString(e));
    addr[dev] = p;
    ctx_of[dev] = current_context_id();  // the lookup has created the context if needed
  }
  *out = addr[dev];
  return D2SD_OK;
}

}  // namespace
}  // namespace d2sd

extern "C" int d2sd_verify_accept_noalloc(const void* logits, int32_t dtype,
                                          int32_t num_branches, int32_t block_len, int64_t vocab,
                                          int64_t stride_branch, int64_t stride_pos,
                                          const int64_t* block_ids, int64_t ids_stride_branch,
                                          int64_t ids_stride_pos, int32_t* result,
                                          int64_t* accepted_ids, int64_t* argmax_out,
                                          void* stream) {
  using namespace d2sd;
  if (num_branches <= 0 || block_len <= 0 || vocab <= 0)
    return fail(D2SD_ERR_INVALID_ARGUMENT, "d2sd_verify_accept_noalloc: invalid argument");
  const int64_t need =
      workspace_bytes(static_cast<int64_t>(num_branches) * block_len, accept_grid());
  if (need > kStaticScratchBytes)
    return fail(D2SD_ERR_UNSUPPORTED,
                "d2sd_verify_accept_noalloc: this shape needs " + std::to_string(need) +
                    " bytes of scratch; the static scratch array holds " +
                    std::to_string(kStaticScratchBytes));
  void* scratch = nullptr;
  int rc = static_scratch(&scratch);
  if (rc) return rc;
  // the completion ticket must start at zero (256 bytes at the array's start)
  cudaError_t e = cudaMemsetAsync(scratch, 0, 256, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess)
    return fail(D2SD_ERR_CUDA, std::string("cudaMemsetAsync: ") + cudaGetErrorString(e));
  return d2sd_verify_accept(logits, dtype, num_branches, block_len, vocab, stride_branch,
                            stride_pos, block_ids, ids_stride_branch, ids_stride_pos, result,
                            accepted_ids, argmax_out, scratch, kStaticScratchBytes, stream);
}
