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
// 16-byte loads, HBM-bound) and the walk then runs on one warp with a ballot
// per step. The winning branch returned is vb of the last iteration, the branch
// whose logits produced the bonus token and whose K/V the commit appends
// (generation/d3_generator.py:229-230).
// Ties resolve to the first maximal index and NaN counts as maximal (first NaN
// wins), the torch.argmax convention.
//
// Grid: (chunks, rows). Each CTA reduces one chunk of one row to (value, index)
// and the last CTA to finish (atomic ticket) reduces the chunks and walks.
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

__host__ __device__ inline int num_chunks_for(int64_t rows, int64_t vocab, int sms) {
  // ~8 CTAs per SM over the whole grid, chunks of at least 8192 elements.
  int64_t target = (static_cast<int64_t>(sms) * 8 + rows - 1) / rows;
  int64_t max_by_size = (vocab + 8191) / 8192;
  int64_t c = target < max_by_size ? target : max_by_size;
  if (c < 1) c = 1;
  if (c > 64) c = 64;
  return static_cast<int>(c);
}

struct Workspace {
  unsigned int* ticket;  // 1 word, zero between launches
  float* pval;           // [rows][chunks]
  int64_t* pidx;         // [rows][chunks]
  int64_t* amax;         // [rows]
};

__host__ __device__ inline int64_t align_up(int64_t x, int64_t a) { return (x + a - 1) / a * a; }

__host__ __device__ inline int64_t workspace_bytes(int64_t rows, int chunks) {
  return 256 + align_up(rows * chunks * 4, 256) + align_up(rows * chunks * 8, 256) +
         align_up(rows * 8, 256);
}

__host__ __device__ inline Workspace carve(void* base, int64_t rows, int chunks) {
  uint8_t* b = static_cast<uint8_t*>(base);
  Workspace w;
  w.ticket = reinterpret_cast<unsigned int*>(b);
  b += 256;
  w.pval = reinterpret_cast<float*>(b);
  b += align_up(rows * chunks * 4, 256);
  w.pidx = reinterpret_cast<int64_t*>(b);
  b += align_up(rows * chunks * 8, 256);
  w.amax = reinterpret_cast<int64_t*>(b);
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
};
template <>
struct VecMax<__half> {
  static __device__ __forceinline__ float max(const uint4& v) {
    const uint32_t m = max_nan_f16x2(max_nan_f16x2(v.x, v.y), max_nan_f16x2(v.z, v.w));
    const __half2 h = *reinterpret_cast<const __half2*>(&m);
    return max_nan(__low2float(h), __high2float(h));
  }
};

template <typename T>
__global__ void __launch_bounds__(kThreads)
    accept_kernel(const T* __restrict__ logits, int B, int TB, int64_t V, int64_t s_b,
                  int64_t s_t, const int64_t* __restrict__ ids, int64_t ids_sb, int64_t ids_st,
                  int32_t* result, int64_t* accepted, int64_t* argmax_out, Workspace ws,
                  int chunks) {
  constexpr int VN = Vec<T>::N;
  __shared__ float sv[kThreads / 32];
  __shared__ int64_t si[kThreads / 32];
  __shared__ bool last;
  const int row = blockIdx.y;
  const int chunk = blockIdx.x;
  const int b = row / TB, t = row % TB;
  const T* base = logits + static_cast<int64_t>(b) * s_b + static_cast<int64_t>(t) * s_t;
  const int64_t csize = ((V + chunks - 1) / chunks + VN - 1) / VN * VN;
  const int64_t c0 = static_cast<int64_t>(chunk) * csize;
  const int64_t c1 = c0 + csize < V ? c0 + csize : V;

  // Per-thread scan in increasing index order. Each 16-byte vector is reduced
  // with a NaN-propagating max first; only a vector that beats the running best
  // (or holds a NaN) is searched for its first maximal index. A strict ">"
  // keeps the first index among equal maxima; once the best is NaN nothing
  // replaces it (torch.argmax: the first NaN wins).
  float best_v = -INFINITY;
  int64_t best_i = INT64_MAX;
  if (c0 < c1) {
    const bool vec_ok = (reinterpret_cast<uintptr_t>(base + c0) & 15u) == 0;
    const int64_t nvec = vec_ok ? (c1 - c0) / VN : 0;
    const int64_t tail0 = c0 + nvec * VN;
    const uint4* src = reinterpret_cast<const uint4*>(base + c0);
    if (threadIdx.x < nvec) best_i = c0 + static_cast<int64_t>(threadIdx.x) * VN;
    auto visit = [&](const uint4& raw, int64_t first) {
      const float vm = VecMax<T>::max(raw);
      if (!(vm <= best_v) && best_v == best_v) {
        const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
        for (int k = 0; k < VN; ++k) {
          const float x = Num<T>::to_f(e[k]);
          if (x != x || x == vm) {
            best_v = x;
            best_i = first + k;
            break;
          }
        }
      }
    };
    int64_t vI = threadIdx.x;
    for (; vI + 3 * kThreads < nvec; vI += 4 * kThreads) {
      uint4 raw[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) raw[u] = __ldg(src + vI + u * kThreads);
#pragma unroll
      for (int u = 0; u < 4; ++u) visit(raw[u], c0 + (vI + u * kThreads) * VN);
    }
    for (; vI < nvec; vI += kThreads) visit(__ldg(src + vI), c0 + vI * VN);
    for (int64_t j = tail0 + threadIdx.x; j < c1; j += kThreads) {
      const float x = Num<T>::to_f(base[j]);
      if (best_i == INT64_MAX) {
        best_v = x;
        best_i = j;
      } else if ((x > best_v || (x != x)) && best_v == best_v) {
        best_v = x;
        best_i = j;
      }
    }
  }
  // block reduce
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best_v, o);
    const int64_t oi = __shfl_xor_sync(0xffffffffu, best_i, o);
    if (better(ov, oi, best_v, best_i)) {
      best_v = ov;
      best_i = oi;
    }
  }
  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
  if (lane == 0) {
    sv[warp] = best_v;
    si[warp] = best_i;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < kThreads / 32; ++w) {
      if (better(sv[w], si[w], best_v, best_i)) {
        best_v = sv[w];
        best_i = si[w];
      }
    }
    ws.pval[static_cast<int64_t>(row) * chunks + chunk] = best_v;
    ws.pidx[static_cast<int64_t>(row) * chunks + chunk] = best_i;
    __threadfence();
    const unsigned total = gridDim.x * gridDim.y;
    last = atomicAdd(ws.ticket, 1u) == total - 1;
  }
  __syncthreads();
  if (!last) return;
  __threadfence();

  // ---- last CTA: per-row argmax over chunks ----
  const int rows = B * TB;
  for (int r = threadIdx.x; r < rows; r += kThreads) {
    float bv = -INFINITY;
    int64_t bi = INT64_MAX;
    for (int c = 0; c < chunks; ++c) {
      const float v = ws.pval[static_cast<int64_t>(r) * chunks + c];
      const int64_t ix = ws.pidx[static_cast<int64_t>(r) * chunks + c];
      if (better(v, ix, bv, bi)) {
        bv = v;
        bi = ix;
      }
    }
    if (bi == INT64_MAX) bi = 0;  // row of only -inf: torch returns 0
    ws.amax[r] = bi;
    if (argmax_out) argmax_out[r] = bi;
  }
  __syncthreads();

  // ---- the acceptance walk on warp 0 ----
  if (warp == 0) {
    // valid set as a 64-bit mask; lane l owns branches l and l + 32
    uint64_t valid = (B >= 64) ? ~0ull : ((1ull << B) - 1ull);
    int acc = 0;
    int vb = 0;
    while (true) {
      vb = __ffsll(static_cast<long long>(valid)) - 1;
      const int64_t tok = ws.amax[vb * TB + acc];
      if (lane == 0) accepted[acc] = tok;
      acc += 1;
      if (acc == TB) break;
      bool m0 = false, m1 = false;
      if (lane < B) m0 = ids[lane * ids_sb + acc * ids_st] == tok;
      if (lane + 32 < B) m1 = ids[(lane + 32) * ids_sb + acc * ids_st] == tok;
      const uint64_t match = static_cast<uint64_t>(__ballot_sync(0xffffffffu, m0)) |
                             (static_cast<uint64_t>(__ballot_sync(0xffffffffu, m1)) << 32);
      valid &= match;
      if (valid == 0) break;
    }
    for (int k = acc + lane; k < TB; k += 32) accepted[k] = -1;
    if (lane == 0) {
      result[0] = acc;
      result[1] = vb;
      *ws.ticket = 0u;  // leave the workspace ready for the next launch
    }
  }
}

}  // namespace
}  // namespace d2sd

extern "C" int64_t d2sd_verify_accept_workspace_size(int32_t num_branches, int32_t block_len,
                                                     int64_t vocab) {
  if (num_branches <= 0 || block_len <= 0 || vocab <= 0) return -1;
  const int64_t rows = static_cast<int64_t>(num_branches) * block_len;
  const int chunks = d2sd::num_chunks_for(rows, vocab, d2sd::current_sm_count());
  return d2sd::workspace_bytes(rows, chunks);
}

extern "C" int d2sd_verify_accept(const void* logits, int32_t dtype, int32_t num_branches,
                                  int32_t block_len, int64_t vocab, int64_t stride_branch,
                                  int64_t stride_pos, const int64_t* block_ids,
                                  int64_t ids_stride_branch, int64_t ids_stride_pos,
                                  int32_t* result, int64_t* accepted_ids, int64_t* argmax_out,
                                  void* workspace, int64_t workspace_bytes, void* stream) {
  using namespace d2sd;
  if (!logits || !block_ids || !result || !accepted_ids || !workspace || num_branches <= 0 ||
      block_len <= 0 || vocab <= 0)
    return fail(D2SD_ERR_INVALID_ARGUMENT, "d2sd_verify_accept: invalid argument");
  if (num_branches > kMaxBranches)
    return fail(D2SD_ERR_UNSUPPORTED, "d2sd_verify_accept: at most 64 branches");
  const int64_t rows = static_cast<int64_t>(num_branches) * block_len;
  if (rows > 65535)
    return fail(D2SD_ERR_UNSUPPORTED, "d2sd_verify_accept: too many logits rows");
  const int chunks = num_chunks_for(rows, vocab, current_sm_count());
  if (workspace_bytes < d2sd::workspace_bytes(rows, chunks))
    return fail(D2SD_ERR_WORKSPACE, "d2sd_verify_accept: workspace too small");
  if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0)
    return fail(D2SD_ERR_INVALID_ARGUMENT, "d2sd_verify_accept: workspace must be 256-byte aligned");
  Workspace ws = carve(workspace, rows, chunks);
  dim3 grid(chunks, static_cast<unsigned>(rows));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case D2SD_DTYPE_F32:
      accept_kernel<float><<<grid, kThreads, 0, st>>>(
          static_cast<const float*>(logits), num_branches, block_len, vocab, stride_branch,
          stride_pos, block_ids, ids_stride_branch, ids_stride_pos, result, accepted_ids,
          argmax_out, ws, chunks);
      break;
    case D2SD_DTYPE_BF16:
      accept_kernel<__nv_bfloat16><<<grid, kThreads, 0, st>>>(
          static_cast<const __nv_bfloat16*>(logits), num_branches, block_len, vocab,
          stride_branch, stride_pos, block_ids, ids_stride_branch, ids_stride_pos, result,
          accepted_ids, argmax_out, ws, chunks);
      break;
    case D2SD_DTYPE_F16:
      accept_kernel<__half><<<grid, kThreads, 0, st>>>(
          static_cast<const __half*>(logits), num_branches, block_len, vocab, stride_branch,
          stride_pos, block_ids, ids_stride_branch, ids_stride_pos, result, accepted_ids,
          argmax_out, ws, chunks);
      break;
    default:
      return fail(D2SD_ERR_UNSUPPORTED, "d2sd_verify_accept: unknown dtype");
  }
  return check_launch("accept_kernel");
}
