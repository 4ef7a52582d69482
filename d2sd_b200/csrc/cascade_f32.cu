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
// A CTA takes 16 query rows of one kv head (row = token * G + g, the G query
// heads of the kv head) and walks the keys in tiles of 32: the prefix keys
// [kv_start, P), then the block tokens of the blocks its rows' tokens lie in.
// Each tile's K and V rows are staged in shared memory by 16-byte cp.async
// copies, one tile ahead of the one being computed. Per tile, a warp (4 rows)
// computes the 4 x 32 scores with lane = key (Q broadcast from shared memory),
// updates each row's online softmax (max and sum across the warp), and adds
// P.V with lane = 4 dims (P broadcast by shuffle). All in fp32 with expf.
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

constexpr int kF32Rows = 16;     // query rows per CTA (4 per warp)
constexpr int kF32Keys = 32;     // keys per tile (one per lane in Q.K^T)
constexpr int kF32Threads = 128;

template <int D>
struct F32Smem {
  static constexpr int KS = D + 4;  // K row stride: 16-byte rows, conflict-free float4 reads
  static constexpr int kQ = kF32Rows * D;
  static constexpr int kK = kF32Keys * KS;
  static constexpr int kV = kF32Keys * D;
  static constexpr int kStage = kK + kV;
  static constexpr size_t kBytes = sizeof(float) * (kQ + 2 * kStage);
};

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_0() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

template <int D>
__global__ void __launch_bounds__(kF32Threads) cascade_f32_kernel(const F32Params p, int aligned) {
  using S = F32Smem<D>;
  constexpr int DW = D / 32;  // dims per lane in P.V and the output
  extern __shared__ __align__(16) float sm[];
  float* Qs = sm;
  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
  const int hk = blockIdx.y;
  const int rows_hk = p.num_tokens * p.G;  // rows of this kv head
  const int row0 = blockIdx.x * kF32Rows;

  // ---- Q rows of the CTA, pre-scaled (rows past the end are zero) ----
  for (int e = threadIdx.x; e < kF32Rows * D; e += kF32Threads) {
    const int i = e / D, d = e - (e / D) * D;
    const int r = row0 + i;
    float x = 0.f;
    if (r < rows_hk) {
      const int tok = r / p.G, hq = hk * p.G + (r - (r / p.G) * p.G);
      x = p.q[static_cast<int64_t>(tok) * p.q_st + static_cast<int64_t>(hq) * p.q_sh + d] * p.scale;
    }
    Qs[e] = x;
  }

  // ---- the key tiles: prefix keys, then the block tokens of the CTA's blocks ----
  const int r_last = min(row0 + kF32Rows, rows_hk) - 1;
  const int tok_first = row0 / p.G, tok_last = r_last / p.G;
  const int TB = p.block_len;
  const int n_pre = p.kp ? p.P - p.kv_start : 0;
  const int loc0 = p.kl ? (tok_first / TB) * TB : 0;
  const int loc1 = p.kl ? min((tok_last / TB + 1) * TB, p.num_tokens) : 0;
  const int t_pre = (n_pre + kF32Keys - 1) / kF32Keys;
  const int t_all = t_pre + (loc1 - loc0 + kF32Keys - 1) / kF32Keys;

  // stage tile t (K rows at stride KS, V rows at stride D); keys past the end
  // load a valid key instead (finite values; their P is 0)
  auto stage = [&](int t, int buf) {
    float* Kd = sm + S::kQ + buf * S::kStage;
    float* Vd = Kd + S::kK;
    const float *kb, *vb;
    int64_t st, first;
    int n;
    if (t < t_pre) {
      kb = p.kp; vb = p.vp; st = p.p_st;
      first = p.kv_start + static_cast<int64_t>(t) * kF32Keys;
      n = min(kF32Keys, p.P - static_cast<int>(first));
      kb += static_cast<int64_t>(hk) * p.p_sh;
      vb += static_cast<int64_t>(hk) * p.p_sh;
    } else {
      kb = p.kl; vb = p.vl; st = p.l_st;
      first = loc0 + static_cast<int64_t>(t - t_pre) * kF32Keys;
      n = min(kF32Keys, loc1 - static_cast<int>(first));
      kb += static_cast<int64_t>(hk) * p.l_sh;
      vb += static_cast<int64_t>(hk) * p.l_sh;
    }
    constexpr int CH = D / 4;  // 16-byte chunks per row
    for (int e = threadIdx.x; e < kF32Keys * CH; e += kF32Threads) {
      const int j = e / CH, c = e - (e / CH) * CH;
      const int64_t key = first + min(j, n - 1);
      const float* ks = kb + key * st + 4 * c;
      const float* vs = vb + key * st + 4 * c;
      if (aligned) {
        cp_async16(Kd + j * S::KS + 4 * c, ks);
        cp_async16(Vd + j * D + 4 * c, vs);
      } else {
#pragma unroll
        for (int w = 0; w < 4; ++w) {
          Kd[j * S::KS + 4 * c + w] = ks[w];
          Vd[j * D + 4 * c + w] = vs[w];
        }
      }
    }
    cp_async_commit();
  };

  // per row of the warp: token, its block / position, allowed local keys
  int tok_i[4], blk_i[4];
  uint64_t allow_i[4];
  bool live_i[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = row0 + warp * 4 + i;
    live_i[i] = r < rows_hk;
    const int tok = live_i[i] ? r / p.G : 0;
    tok_i[i] = tok;
    blk_i[i] = tok / TB;
    const int tt = tok - (tok / TB) * TB;
    uint64_t a = ~0ull;
    if (p.mask_mode == D2SD_MASK_CAUSAL) a = (tt >= 63) ? ~0ull : ((2ull << tt) - 1ull);
    else if (p.mask_mode == D2SD_MASK_CUSTOM && p.kl && live_i[i]) a = p.custom_mask[tok];
    allow_i[i] = a;
  }
  float m_i[4], l_i[4], acc[4][DW];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    m_i[i] = -INFINITY;
    l_i[i] = 0.f;
#pragma unroll
    for (int c = 0; c < DW; ++c) acc[i][c] = 0.f;
  }

  if (t_all > 0) stage(0, 0);
  for (int t = 0; t < t_all; ++t) {
    const int buf = t & 1;
    if (t + 1 < t_all) {
      stage(t + 1, buf ^ 1);  // the next tile's copies run during this tile
      cp_async_wait_1();
    } else {
      cp_async_wait_0();
    }
    __syncthreads();  // tile t (and, at t = 0, Q) visible to every warp
    const float* Kt = sm + S::kQ + buf * S::kStage;
    const float* Vt = Kt + S::kK;
    // scores of the warp's 4 rows against key `lane`
    float s[4] = {0.f, 0.f, 0.f, 0.f};
    const float* kr = Kt + lane * S::KS;
    const float* q0 = Qs + (warp * 4) * D;
#pragma unroll 8
    for (int d = 0; d < D; d += 4) {
      const float4 k4 = *reinterpret_cast<const float4*>(kr + d);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float4 q4 = *reinterpret_cast<const float4*>(q0 + i * D + d);
        s[i] = fmaf(q4.x, k4.x, s[i]);
        s[i] = fmaf(q4.y, k4.y, s[i]);
        s[i] = fmaf(q4.z, k4.z, s[i]);
        s[i] = fmaf(q4.w, k4.w, s[i]);
      }
    }
    // which (row, key) pairs count
    bool valid[4];
    if (t < t_pre) {
      const bool in = t * kF32Keys + lane < n_pre;
#pragma unroll
      for (int i = 0; i < 4; ++i) valid[i] = in && live_i[i];
    } else {
      const int key = loc0 + (t - t_pre) * kF32Keys + lane;
      const int kb = key / TB, kt = key - (key / TB) * TB;
#pragma unroll
      for (int i = 0; i < 4; ++i)
        valid[i] = live_i[i] && key < loc1 && kb == blk_i[i] && ((allow_i[i] >> kt) & 1ull);
    }
    float pr[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float tmax = valid[i] ? s[i] : -INFINITY;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, o));
      const float mn = fmaxf(m_i[i], tmax);
      const float alpha = (m_i[i] == -INFINITY) ? 0.f : expf(m_i[i] - mn);
      pr[i] = valid[i] ? expf(s[i] - mn) : 0.f;
      float ps = pr[i];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
      l_i[i] = fmaf(l_i[i], alpha, ps);
#pragma unroll
      for (int c = 0; c < DW; ++c) acc[i][c] *= alpha;
      m_i[i] = mn;
    }
    // P.V: lane holds dims lane + 32 c
#pragma unroll 4
    for (int j = 0; j < kF32Keys; ++j) {
      float vv[DW];
#pragma unroll
      for (int c = 0; c < DW; ++c) vv[c] = Vt[j * D + lane + 32 * c];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float pj = __shfl_sync(0xffffffffu, pr[i], j);
#pragma unroll
        for (int c = 0; c < DW; ++c) acc[i][c] = fmaf(pj, vv[c], acc[i][c]);
      }
    }
    __syncthreads();  // every warp is done with this buffer before it is refilled
  }

  // ---- per row: normalise, merge with a dense prefix state, sinks, store ----
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if (!live_i[i]) continue;
    const int r = row0 + warp * 4 + i;
    const int tok = tok_i[i], hq = hk * p.G + (r - (r / p.G) * p.G);
    const float l = l_i[i], m = m_i[i];
    float lse2 = (l > 0.f) ? (m + logf(l)) * kLog2e : -INFINITY;
    const float inv = (l > 0.f) ? 1.f / l : 0.f;
    float o[DW];
#pragma unroll
    for (int c = 0; c < DW; ++c) o[c] = acc[i][c] * inv;
    if (p.prefix_out) {
      // merge_state_in_place((prefix_out, prefix_lse), (o, lse2)), base 2
      const float lp = p.prefix_lse[static_cast<int64_t>(tok) * p.pl_st + hq];
      const float M = fmaxf(lp, lse2);
      const float wa = (lp == -INFINITY) ? 0.f : exp2f(lp - M);
      const float wb = (lse2 == -INFINITY) ? 0.f : exp2f(lse2 - M);
      const float den = wa + wb;
      const float* po = p.prefix_out + static_cast<int64_t>(tok) * p.po_st +
                        static_cast<int64_t>(hq) * p.po_sh;
#pragma unroll
      for (int c = 0; c < DW; ++c)
        o[c] = den > 0.f ? (wa * po[lane + 32 * c] + wb * o[c]) / den : 0.f;
      lse2 = den > 0.f ? M + log2f(den) : -INFINITY;
    }
    float factor = 1.f;
    if (p.sinks && p.sink_mode != D2SD_SINK_NONE) {
      const float x = (p.sink_mode == D2SD_SINK_EXACT ? lse2 * kLn2 : lse2) - p.sinks[hq];
      factor = 1.f / (1.f + expf(-x));
    }
    float* orow = p.out + static_cast<int64_t>(tok) * p.o_st + static_cast<int64_t>(hq) * p.o_sh;
#pragma unroll
    for (int c = 0; c < DW; ++c) orow[lane + 32 * c] = o[c] * factor;
    if (lane == 0 && p.lse) p.lse[static_cast<int64_t>(tok) * p.lse_st + hq] = lse2;
  }
}

template <int D>
int launch_f32(const F32Params& prm, int num_kv_heads, cudaStream_t st) {
  using S = F32Smem<D>;
  static int configured = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured != dev) {
    cudaError_t e = cudaFuncSetAttribute(cascade_f32_kernel<D>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(S::kBytes));
    if (e != cudaSuccess)
      return fail(D2SD_ERR_CUDA, std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e));
    configured = dev;
  }
  // 16-byte copies need 16-byte aligned rows
  auto al = [](const void* ptr, int64_t a, int64_t b) {
    return ptr == nullptr ||
           ((reinterpret_cast<uintptr_t>(ptr) & 15u) == 0 && a % 4 == 0 && b % 4 == 0);
  };
  const int aligned = al(prm.kp, prm.p_st, prm.p_sh) && al(prm.vp, prm.p_st, prm.p_sh) &&
                      al(prm.kl, prm.l_st, prm.l_sh) && al(prm.vl, prm.l_st, prm.l_sh);
  const int64_t rows_hk = static_cast<int64_t>(prm.num_tokens) * prm.G;
  const dim3 grid(static_cast<unsigned>((rows_hk + kF32Rows - 1) / kF32Rows),
                  static_cast<unsigned>(num_kv_heads));
  cascade_f32_kernel<D><<<grid, kF32Threads, S::kBytes, st>>>(prm, aligned);
  return check_launch("cascade_f32_kernel");
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
  if (n * (num_qo_heads / num_kv_heads) > INT32_MAX)
    return fail(D2SD_ERR_UNSUPPORTED, "d2sd_cascade_attention_f32: too many rows");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (head_dim == 128) return launch_f32<128>(prm, num_kv_heads, st);
  if (head_dim == 64) return launch_f32<64>(prm, num_kv_heads, st);
  return launch_f32<32>(prm, num_kv_heads, st);
}
