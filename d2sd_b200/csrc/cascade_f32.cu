// fp32 cascade verify attention (the reference's fp32
// torch.sdpa path at 1e-5 tolerance).
//
// The bf16 kernels (a) and (b) run on the tensor cores and round P and the
// level-1 output to 16 bits, as the reference's FlashInfer kernels do; an
// fp32 model (generation/verification.py with a float32 target, or the
// reference's CPU path) needs fp32 all the way. This kernel computes, for each
// query row, the softmax over the visible prefix keys [kv_start, P) and the
// row's own block tokens (causal, full or a custom bitmask), optionally merged
// with a dense prefix state (the CascadeGraphRunner.run form, model/
// cascade_graph.py:76-112) and rescaled by the GPT-OSS sinks
// (generation/verification.py:173-176), in fp32 with exact expf/logf. The LSE
// it returns is base 2 (FlashInfer's convention, as everywhere in this library).
//
// One warp per (token, query head) row, lane l holding dims l, l+32, ...; an
// online softmax over the keys. The work is small (config 1: 64 rows x 32
// heads x 528 keys), so plain coalesced loads serve.
#include "common.cuh"

namespace d2sd {
namespace {

struct F32Params {
  const float* q;
  int64_t q_st, q_sh;
  const float* kp;  // prefix keys / values [P, Hk, D] (any token/head strides) or NULL
  const float* vp;
  int64_t p_st, p_sh;
  int32_t P, kv_start;
  const float* kl;  // block tokens' keys / values [N, Hk, D] or NULL
  const float* vl;
  int64_t l_st, l_sh;
  int32_t num_tokens, block_len, mask_mode;
  const uint64_t* custom_mask;
  const float* prefix_out;  // dense prefix state [N, Hq, D] / lse [N, Hq] base 2, or NULL
  int64_t po_st, po_sh;
  const float* prefix_lse;
  int64_t pl_st;
  const float* sinks;
  int32_t sink_mode;
  float* out;
  int64_t o_st, o_sh;
  float* lse;
  int64_t lse_st;
  int32_t Hq, G;
  float scale;
};

template <int DW>  // dims per lane: D / 32
__global__ void __launch_bounds__(128) cascade_f32_kernel(const F32Params p) {
  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * 4 + warp;
  if (row >= static_cast<int64_t>(p.num_tokens) * p.Hq) return;
  const int tok = static_cast<int>(row / p.Hq), hq = static_cast<int>(row % p.Hq);
  const int hk = hq / p.G;
  float qv[DW], acc[DW];
  const float* qr = p.q + static_cast<int64_t>(tok) * p.q_st + static_cast<int64_t>(hq) * p.q_sh;
#pragma unroll
  for (int k = 0; k < DW; ++k) {
    qv[k] = qr[lane + 32 * k] * p.scale;
    acc[k] = 0.f;
  }
  float m = -INFINITY, l = 0.f;
  auto visit = [&](const float* kr, const float* vr) {
    float s = 0.f;
#pragma unroll
    for (int k = 0; k < DW; ++k) s = fmaf(qv[k], kr[lane + 32 * k], s);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    const float mn = fmaxf(m, s);
    const float alpha = (m == -INFINITY) ? 0.f : expf(m - mn);
    const float pj = expf(s - mn);
    l = fmaf(l, alpha, pj);
#pragma unroll
    for (int k = 0; k < DW; ++k) acc[k] = fmaf(acc[k], alpha, pj * vr[lane + 32 * k]);
    m = mn;
  };
  if (p.kp) {
    const int64_t hoff = static_cast<int64_t>(hk) * p.p_sh;
    for (int j = p.kv_start; j < p.P; ++j)
      visit(p.kp + j * p.p_st + hoff, p.vp + j * p.p_st + hoff);
  }
  if (p.kl) {
    const int TB = p.block_len;
    const int blk = tok / TB, t = tok - (tok / TB) * TB;
    uint64_t allowed;
    if (p.mask_mode == D2SD_MASK_CAUSAL) allowed = (t >= 63) ? ~0ull : ((2ull << t) - 1ull);
    else if (p.mask_mode == D2SD_MASK_CUSTOM) allowed = p.custom_mask[tok];
    else allowed = ~0ull;
    const int64_t hoff = static_cast<int64_t>(hk) * p.l_sh;
    for (int j = 0; j < TB; ++j) {
      if (!((allowed >> j) & 1ull)) continue;
      const int64_t tj = static_cast<int64_t>(blk) * TB + j;
      visit(p.kl + tj * p.l_st + hoff, p.vl + tj * p.l_st + hoff);
    }
  }
  // this part's state: normalised output and base-2 LSE
  float lse2 = (l > 0.f) ? (m + logf(l)) * kLog2e : -INFINITY;
  const float inv = (l > 0.f) ? 1.f / l : 0.f;
#pragma unroll
  for (int k = 0; k < DW; ++k) acc[k] *= inv;
  if (p.prefix_out) {
    // merge_state_in_place((prefix_out, prefix_lse), (acc, lse2)), base 2
    const float lp = p.prefix_lse[static_cast<int64_t>(tok) * p.pl_st + hq];
    const float M = fmaxf(lp, lse2);
    const float wa = (lp == -INFINITY) ? 0.f : exp2f(lp - M);
    const float wb = (lse2 == -INFINITY) ? 0.f : exp2f(lse2 - M);
    const float den = wa + wb;
    const float* po = p.prefix_out + static_cast<int64_t>(tok) * p.po_st +
                      static_cast<int64_t>(hq) * p.po_sh;
#pragma unroll
    for (int k = 0; k < DW; ++k)
      acc[k] = den > 0.f ? (wa * po[lane + 32 * k] + wb * acc[k]) / den : 0.f;
    lse2 = den > 0.f ? M + log2f(den) : -INFINITY;
  }
  float factor = 1.f;
  if (p.sinks && p.sink_mode != D2SD_SINK_NONE) {
    const float x = (p.sink_mode == D2SD_SINK_EXACT ? lse2 * kLn2 : lse2) - p.sinks[hq];
    factor = 1.f / (1.f + expf(-x));
  }
  float* orow = p.out + static_cast<int64_t>(tok) * p.o_st + static_cast<int64_t>(hq) * p.o_sh;
#pragma unroll
  for (int k = 0; k < DW; ++k) orow[lane + 32 * k] = acc[k] * factor;
  if (lane == 0 && p.lse) p.lse[static_cast<int64_t>(tok) * p.lse_st + hq] = lse2;
}

}  // namespace
}  // namespace d2sd

extern "C" int d2sd_cascade_attention_f32(
    const float* q, int64_t q_stride_token, int64_t q_stride_head, const float* k_prefix,
    const float* v_prefix, int64_t prefix_stride_token, int64_t prefix_stride_head,
    int32_t prefix_len, int32_t kv_start, const float* k_local, const float* v_local,
    int64_t local_stride_token, int64_t local_stride_head, int32_t num_blocks,
    int32_t block_len, int32_t mask_mode, const uint64_t* custom_mask, const float* prefix_out,
    int64_t prefix_out_stride_token, int64_t prefix_out_stride_head, const float* prefix_lse,
    int64_t prefix_lse_stride_token, const float* sinks, int32_t sink_mode, float* out,
    int64_t out_stride_token, int64_t out_stride_head, float* lse, int64_t lse_stride_token,
    int32_t num_qo_heads, int32_t num_kv_heads, int32_t head_dim, float sm_scale, void* stream) {
  using namespace d2sd;
  if (!q || !out || num_blocks < 0 || block_len <= 0 || num_qo_heads <= 0 ||
      num_kv_heads <= 0 || num_qo_heads % num_kv_heads || prefix_len < 0 || kv_start < 0 ||
      kv_start > prefix_len || (prefix_len > 0 && (!k_prefix || !v_prefix)) ||
      ((k_local == nullptr) != (v_local == nullptr)) || (prefix_out && !prefix_lse))
    return fail(D2SD_ERR_INVALID_ARGUMENT, "d2sd_cascade_attention_f32: invalid argument");
  if (mask_mode < D2SD_MASK_NONE || mask_mode > D2SD_MASK_CUSTOM ||
      (mask_mode == D2SD_MASK_CUSTOM && k_local && !custom_mask))
    return fail(D2SD_ERR_INVALID_ARGUMENT, "d2sd_cascade_attention_f32: invalid mask");
  if (k_local && block_len > 64)
    return fail(D2SD_ERR_UNSUPPORTED, "d2sd_cascade_attention_f32: block_len must be <= 64");
  if (head_dim != 32 && head_dim != 64 && head_dim != 128)
    return fail(D2SD_ERR_UNSUPPORTED, "d2sd_cascade_attention_f32: head_dim must be 32, 64 or 128");
  const int64_t n = static_cast<int64_t>(num_blocks) * block_len;
  if (n == 0) return D2SD_OK;
  if (n > INT32_MAX)
    return fail(D2SD_ERR_UNSUPPORTED, "d2sd_cascade_attention_f32: too many tokens");
  F32Params prm;
  prm.q = q;
  prm.q_st = q_stride_token;
  prm.q_sh = q_stride_head;
  prm.kp = prefix_len > 0 ? k_prefix : nullptr;
  prm.vp = v_prefix;
  prm.p_st = prefix_stride_token;
  prm.p_sh = prefix_stride_head;
  prm.P = prefix_len;
  prm.kv_start = kv_start;
  prm.kl = k_local;
  prm.vl = v_local;
  prm.l_st = local_stride_token;
  prm.l_sh = local_stride_head;
  prm.num_tokens = static_cast<int32_t>(n);
  prm.block_len = block_len;
  prm.mask_mode = mask_mode;
  prm.custom_mask = custom_mask;
  prm.prefix_out = prefix_out;
  prm.po_st = prefix_out_stride_token;
  prm.po_sh = prefix_out_stride_head;
  prm.prefix_lse = prefix_lse;
  prm.pl_st = prefix_lse_stride_token;
  prm.sinks = sinks;
  prm.sink_mode = sink_mode;
  prm.out = out;
  prm.o_st = out_stride_token;
  prm.o_sh = out_stride_head;
  prm.lse = lse;
  prm.lse_st = lse_stride_token;
  prm.Hq = num_qo_heads;
  prm.G = num_qo_heads / num_kv_heads;
  prm.scale = sm_scale;
  const int64_t rows = n * num_qo_heads;
  const dim3 grid(static_cast<unsigned>((rows + 3) / 4));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (head_dim == 128) cascade_f32_kernel<4><<<grid, 128, 0, st>>>(prm);
  else if (head_dim == 64) cascade_f32_kernel<2><<<grid, 128, 0, st>>>(prm);
  else cascade_f32_kernel<1><<<grid, 128, 0, st>>>(prm);
  return check_launch("cascade_f32_kernel");
}
