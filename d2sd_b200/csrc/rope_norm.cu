// The step before the verify attention, fused: per-head RMSNorm of the block's
// q and k (Qwen3's QK-norm) and the rotary embedding, in one launch for q and k.
//
// Reference: generation/verification.py:113-124 (q_norm / k_norm, then
// rope_apply), with _apply_rotary_pos_emb_qwen3 (:21-28) and
// _apply_rotary_pos_emb_gpt_oss (:31-43); the norm is transformers'
// Qwen3RMSNorm.forward (x.float() * rsqrt(mean(x^2) + eps), cast to the input
// dtype, times the weight). Every rounding to the 16-bit dtype that those eager
// torch expressions make is made here too, in the same order:
//   n = rnd(x * rsqrt(var + eps));  y = rnd(w * n)              (norm)
//   out = rnd(rnd(y * cos) + rnd(rot(y) * sin)),  rot(y) = cat(-y2, y1)
// The two RoPE forms are the same expression: GPT-OSS's
// (first*cos - second*sin, second*cos + first*sin) with a half-width table is
// rotate_half with the table's halves repeated, and a - b = a + (-b) exactly.
// So cos/sin are read as [positions, head_dim/2] tables (a Qwen3 full-width
// table, whose halves are equal, is read through its first half).
//
// One warp per (token, head) row, head_dim/32 consecutive elements per lane;
// lanes l and l ^ 16 hold the two halves of the row (the rotate_half partner).
#include "common.cuh"

namespace d2sd {
namespace {

template <typename T>
__device__ __forceinline__ float rnd(float x) {
  return Num<T>::to_f(Num<T>::from_f(x));
}

struct RopeSide {
  const void* in;
  void* out;
  int64_t in_st, in_sh, out_st, out_sh;  // element strides (token, head)
  const void* weight;                    // [head_dim] norm weight, or nullptr
  int heads;
};

template <typename T, int D>
__global__ void __launch_bounds__(256)
    qk_norm_rope_kernel(RopeSide qs, RopeSide ks, int ntok, int block_len, float eps, int norm,
                        const T* __restrict__ cos_t, const T* __restrict__ sin_t,
                        int64_t cs_stride, const int32_t* __restrict__ positions) {
  constexpr int E = D / 32;  // elements per lane
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + threadIdx.x / 32;
  const int64_t rows_q = static_cast<int64_t>(ntok) * qs.heads;
  const int64_t rows = rows_q + static_cast<int64_t>(ntok) * ks.heads;
  if (row >= rows) return;  // warp-uniform
  const bool isq = row < rows_q;
  const RopeSide& sd = isq ? qs : ks;
  const int64_t r = isq ? row : row - rows_q;
  const int tok = static_cast<int>(r / sd.heads);
  const int h = static_cast<int>(r % sd.heads);
  const int pos = positions ? positions[tok % block_len] : tok % block_len;
  const T* src = static_cast<const T*>(sd.in) + tok * sd.in_st + h * sd.in_sh + lane * E;
  T* dst = static_cast<T*>(sd.out) + tok * sd.out_st + h * sd.out_sh + lane * E;
  float y[E];
#pragma unroll
  for (int e = 0; e < E; ++e) y[e] = Num<T>::to_f(src[e]);
  if (norm) {
    float ss = 0.f;
#pragma unroll
    for (int e = 0; e < E; ++e) ss = fmaf(y[e], y[e], ss);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float inv = rsqrtf(ss / static_cast<float>(D) + eps);
    const T* w = static_cast<const T*>(sd.weight) + lane * E;
#pragma unroll
    for (int e = 0; e < E; ++e) y[e] = rnd<T>(Num<T>::to_f(w[e]) * rnd<T>(y[e] * inv));
  }
  const bool first_half = lane < 16;
  const int c0 = (lane & 15) * E;  // column inside the half-width table
  const T* ct = cos_t + static_cast<int64_t>(pos) * cs_stride + c0;
  const T* st = sin_t + static_cast<int64_t>(pos) * cs_stride + c0;
#pragma unroll
  for (int e = 0; e < E; ++e) {
    const float other = __shfl_xor_sync(0xffffffffu, y[e], 16);
    const float rot = first_half ? -other : other;
    const float a = rnd<T>(y[e] * Num<T>::to_f(ct[e]));
    const float b = rnd<T>(rot * Num<T>::to_f(st[e]));
    dst[e] = Num<T>::from_f(a + b);
  }
}

}  // namespace
}  // namespace d2sd

extern "C" int d2sd_qk_norm_rope(const void* q_in, int64_t q_in_stride_token,
                                 int64_t q_in_stride_head, void* q_out, int64_t q_out_stride_token,
                                 int64_t q_out_stride_head, const void* k_in,
                                 int64_t k_in_stride_token, int64_t k_in_stride_head, void* k_out,
                                 int64_t k_out_stride_token, int64_t k_out_stride_head,
                                 int32_t num_tokens, int32_t num_qo_heads, int32_t num_kv_heads,
                                 int32_t head_dim, int32_t dtype, const void* q_weight,
                                 const void* k_weight, float eps, const void* cos_table,
                                 const void* sin_table, int64_t table_stride, int32_t block_len,
                                 const int32_t* positions, void* stream) {
  using namespace d2sd;
  if (!q_in || !q_out || !k_in || !k_out || !cos_table || !sin_table || num_tokens < 0 ||
      num_qo_heads <= 0 || num_kv_heads <= 0 || block_len <= 0 || table_stride < head_dim / 2)
    return fail(D2SD_ERR_INVALID_ARGUMENT, "d2sd_qk_norm_rope: invalid argument");
  if ((q_weight == nullptr) != (k_weight == nullptr))
    return fail(D2SD_ERR_INVALID_ARGUMENT, "d2sd_qk_norm_rope: give both norm weights or neither");
  if (head_dim != 64 && head_dim != 128)
    return fail(D2SD_ERR_UNSUPPORTED, "d2sd_qk_norm_rope: head_dim must be 64 or 128");
  if (dtype != D2SD_DTYPE_BF16 && dtype != D2SD_DTYPE_F16)
    return fail(D2SD_ERR_UNSUPPORTED, "d2sd_qk_norm_rope: dtype must be bf16 or f16");
  if (num_tokens == 0) return D2SD_OK;
  RopeSide qs{q_in, q_out, q_in_stride_token, q_in_stride_head, q_out_stride_token,
              q_out_stride_head, q_weight, num_qo_heads};
  RopeSide ks{k_in, k_out, k_in_stride_token, k_in_stride_head, k_out_stride_token,
              k_out_stride_head, k_weight, num_kv_heads};
  const int64_t rows = static_cast<int64_t>(num_tokens) * (num_qo_heads + num_kv_heads);
  const dim3 grid(static_cast<unsigned>((rows + 7) / 8));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int norm = q_weight != nullptr;
#define D2SD_ROPE(TT, DD)                                                                    \
  qk_norm_rope_kernel<TT, DD><<<grid, 256, 0, st>>>(qs, ks, num_tokens, block_len, eps, norm, \
                                                    static_cast<const TT*>(cos_table),       \
                                                    static_cast<const TT*>(sin_table),       \
                                                    table_stride, positions)
  if (dtype == D2SD_DTYPE_BF16) {
    if (head_dim == 128) D2SD_ROPE(__nv_bfloat16, 128);
    else D2SD_ROPE(__nv_bfloat16, 64);
  } else {
    if (head_dim == 128) D2SD_ROPE(__half, 128);
    else D2SD_ROPE(__half, 64);
  }
#undef D2SD_ROPE
  return check_launch("qk_norm_rope_kernel");
}
