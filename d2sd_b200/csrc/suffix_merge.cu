// Kernel (b): per-block suffix attention fused with the log-sum-exp merge of
// both cascade levels and the GPT-OSS sink rescale, plus the standalone
// merge_state_in_place replacement.
//
// Reference: CascadeGraphRunner._capture/_run_local_merge
// (model/cascade_graph.py:52-60) runs, per branch i, a causal (verify) or full
// (DTA, model/dflash.py:127-133) single_prefill over the branch's own block
// tokens and then merge_state_in_place into the level-1 state; the sink rescale
// out *= sigmoid(lse - sink) follows at generation/verification.py:173-176.
// Here one launch does all branches: a CTA owns (block, kv head, row chunk),
// stages the block's K/V of that head in shared memory once, and every warp
// walks its query rows (token t, query head g of the group): lane j scores key
// j (and j+32), the warp reduces max/sum with shuffles, lanes own D/32 output
// columns for P.V, and the row is merged in registers with every prefix
// partial state (or with a dense prefix state) before one store.
#include "common.cuh"
#include "plan_layout.h"

namespace d2sd {
namespace {

using namespace plan;

constexpr int kThreads = 128;
constexpr int kWarps = kThreads / 32;
constexpr int kRowsPerCta = 32;
constexpr int kMaxBlockLen = 64;

struct SuffixParams {
  const void* q;
  int64_t q_st, q_sh;
  const void* k;
  const void* v;
  int64_t kv_st, kv_sh;
  int32_t num_blocks, block_len, mask_mode;
  const uint64_t* custom_mask;
  const float* partial;
  const int32_t* plan;
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
  int32_t sink_mode;
  int32_t Hq, Hk, G;
  float scale_log2;
};

template <int DPL>
struct RowState {
  float lse;
  float o[DPL];
};

template <int DPL>
__device__ __forceinline__ void merge_into(RowState<DPL>& a, float lse_b, const float (&ob)[DPL]) {
  if (lse_b == -INFINITY) return;
  if (a.lse == -INFINITY) {
    a.lse = lse_b;
#pragma unroll
    for (int e = 0; e < DPL; ++e) a.o[e] = ob[e];
    return;
  }
  const float M = fmaxf(a.lse, lse_b);
  const float wa = fast_exp2(a.lse - M), wb = fast_exp2(lse_b - M);
  const float inv = 1.f / (wa + wb);
#pragma unroll
  for (int e = 0; e < DPL; ++e) a.o[e] = (wa * a.o[e] + wb * ob[e]) * inv;
  a.lse = M + fast_log2(wa + wb);
}

template <typename T, int D>
__global__ void __launch_bounds__(kThreads) suffix_merge_kernel(const SuffixParams p) {
  constexpr int DPL = D / 32;  // output columns per lane
  constexpr int KP = D + 2;    // padded K row (elements): conflict-free lane-per-key reads
  extern __shared__ __align__(16) uint8_t smem_raw[];
  T* ks = reinterpret_cast<T*>(smem_raw);
  T* vs = ks + kMaxBlockLen * KP;
  float* qbuf = reinterpret_cast<float*>(vs + kMaxBlockLen * D);

  const int blk = blockIdx.x, h = blockIdx.y;
  const int TB = p.block_len, G = p.G;
  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
  const bool has_local = p.k != nullptr;

  if (has_local) {
    const T* kg = static_cast<const T*>(p.k);
    const T* vg = static_cast<const T*>(p.v);
    for (int idx = threadIdx.x; idx < TB * D; idx += kThreads) {
      const int j = idx / D, d = idx % D;
      const int64_t off = (static_cast<int64_t>(blk) * TB + j) * p.kv_st + h * p.kv_sh + d;
      ks[j * KP + d] = kg[off];
      vs[j * D + d] = vg[off];
    }
  }
  __syncthreads();

  const int rows = TB * G;
  const int row_end = min(rows, static_cast<int>(blockIdx.z + 1) * kRowsPerCta);
  float* qw = qbuf + warp * D;
  const T* qg = static_cast<const T*>(p.q);

  for (int r = blockIdx.z * kRowsPerCta + warp; r < row_end; r += kWarps) {
    const int t = r / G, g = r % G;
    const int tok = blk * TB + t;
    const int hq = h * G + g;
    RowState<DPL> st;
    st.lse = -INFINITY;
#pragma unroll
    for (int e = 0; e < DPL; ++e) st.o[e] = 0.f;

    if (has_local) {
      // q row -> per-warp buffer (fp32)
      const T* qrow = qg + static_cast<int64_t>(tok) * p.q_st + static_cast<int64_t>(hq) * p.q_sh;
#pragma unroll
      for (int e = 0; e < DPL; ++e) qw[lane * DPL + e] = Num<T>::to_f(qrow[lane * DPL + e]);
      __syncwarp();
      uint64_t allowed;
      if (p.mask_mode == D2SD_MASK_CAUSAL) {
        allowed = (t >= 63) ? ~0ull : ((2ull << t) - 1ull);
      } else if (p.mask_mode == D2SD_MASK_CUSTOM) {
        allowed = p.custom_mask[tok];
      } else {
        allowed = ~0ull;
      }
      if (TB < 64) allowed &= (1ull << TB) - 1ull;
      float sc[2];
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const int j = lane + half * 32;
        sc[half] = -INFINITY;
        if (j < TB && ((allowed >> j) & 1ull)) {
          const T* kr = ks + j * KP;
          float acc = 0.f;
#pragma unroll 8
          for (int d = 0; d < D; d += 2) {
            acc = fmaf(qw[d], Num<T>::to_f(kr[d]), acc);
            acc = fmaf(qw[d + 1], Num<T>::to_f(kr[d + 1]), acc);
          }
          sc[half] = acc * p.scale_log2;
        }
      }
      float m = fmaxf(sc[0], sc[1]);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      float pj[2];
      pj[0] = sc[0] == -INFINITY ? 0.f : fast_exp2(sc[0] - m);
      pj[1] = sc[1] == -INFINITY ? 0.f : fast_exp2(sc[1] - m);
      float l = pj[0] + pj[1];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
      if (l > 0.f) {
        float acc[DPL];
#pragma unroll
        for (int e = 0; e < DPL; ++e) acc[e] = 0.f;
        const int jmax = TB < 32 ? TB : 32;
        for (int j = 0; j < jmax; ++j) {
          const float pv = __shfl_sync(0xffffffffu, pj[0], j);
          const T* vr = vs + j * D + lane * DPL;
#pragma unroll
          for (int e = 0; e < DPL; ++e) acc[e] = fmaf(pv, Num<T>::to_f(vr[e]), acc[e]);
        }
        for (int j = 32; j < TB; ++j) {
          const float pv = __shfl_sync(0xffffffffu, pj[1], j - 32);
          const T* vr = vs + j * D + lane * DPL;
#pragma unroll
          for (int e = 0; e < DPL; ++e) acc[e] = fmaf(pv, Num<T>::to_f(vr[e]), acc[e]);
        }
        const float inv = 1.f / l;
#pragma unroll
        for (int e = 0; e < DPL; ++e) st.o[e] = acc[e] * inv;
        st.lse = m + fast_log2(l);
      }
      __syncwarp();
    }

    // ---- prefix state ----
    if (p.partial) {
      const int32_t* pl = p.plan;
      const int ptok = p.prefix_token ? p.prefix_token[tok] : tok;
      const int ntok = pl[H_NUM_TOKENS];
      const int req = (ptok >= 0 && ptok < ntok) ? pl[pl[H_OFF_TOKENS] + ptok] : -1;
      if (req >= 0) {
        const int32_t* rq = pl + pl[H_OFF_REQUESTS] + req * kReqInts;
        const int nr = ptok - rq[2];
        const int qrow = nr * G + g;
        const int unit = rq[0] + h * rq[1] + qrow / kTileRows;
        const int32_t* un = pl + pl[H_OFF_UNITS] + unit * kUnitInts;
        const int prow = qrow % kTileRows;
        const int64_t slot_floats = static_cast<int64_t>(kTileRows) * (D + 1);
        for (int s = 0; s < un[1]; ++s) {
          const float* sp = p.partial + static_cast<int64_t>(un[0] + s) * slot_floats;
          const float lse_s = sp[kTileRows * D + prow];
          float ob[DPL];
          const float* orow = sp + prow * D + lane * DPL;
#pragma unroll
          for (int e = 0; e < DPL; ++e) ob[e] = orow[e];
          merge_into<DPL>(st, lse_s, ob);
        }
      }
    } else if (p.prefix_out) {
      const T* po = static_cast<const T*>(p.prefix_out) + static_cast<int64_t>(tok) * p.po_st +
                    static_cast<int64_t>(hq) * p.po_sh + lane * DPL;
      const float lse_p = p.prefix_lse[static_cast<int64_t>(tok) * p.pl_st + hq];
      float ob[DPL];
#pragma unroll
      for (int e = 0; e < DPL; ++e) ob[e] = Num<T>::to_f(po[e]);
      merge_into<DPL>(st, lse_p, ob);
    }

    float factor = 1.f;
    if (p.sinks && p.sink_mode != D2SD_SINK_NONE) {
      const float x = (p.sink_mode == D2SD_SINK_EXACT ? st.lse * kLn2 : st.lse) - p.sinks[hq];
      factor = 1.f / (1.f + __expf(-x));
    }
    T* orow = static_cast<T*>(p.out) + static_cast<int64_t>(tok) * p.o_st +
              static_cast<int64_t>(hq) * p.o_sh + lane * DPL;
#pragma unroll
    for (int e = 0; e < DPL; ++e) orow[e] = Num<T>::from_f(st.o[e] * factor);
    if (lane == 0 && p.lse) p.lse[static_cast<int64_t>(tok) * p.l_st + hq] = st.lse;
  }
}

template <typename T, int D>
int launch_suffix(const SuffixParams& prm, cudaStream_t stream) {
  constexpr int KP = D + 2;
  const size_t smem =
      sizeof(T) * (kMaxBlockLen * KP + kMaxBlockLen * D) + sizeof(float) * kWarps * D;
  static int configured = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured != dev) {
    cudaError_t e = cudaFuncSetAttribute(suffix_merge_kernel<T, D>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess)
      return fail(D2SD_ERR_CUDA, std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e));
    configured = dev;
  }
  const int rows = prm.block_len * prm.G;
  dim3 grid(prm.num_blocks, prm.Hk, (rows + kRowsPerCta - 1) / kRowsPerCta);
  suffix_merge_kernel<T, D><<<grid, kThreads, smem, stream>>>(prm);
  return check_launch("suffix_merge_kernel");
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
                                 int32_t head_dim, int32_t dtype, float sm_scale, void* stream) {
  using namespace d2sd;
  if (!out || num_blocks < 0 || block_len <= 0 || num_qo_heads <= 0 || num_kv_heads <= 0 ||
      num_qo_heads % num_kv_heads != 0)
    return fail(D2SD_ERR_INVALID_ARGUMENT, "d2sd_suffix_merge: invalid argument");
  if (num_blocks == 0) return D2SD_OK;
  if (block_len > kMaxBlockLen)
    return fail(D2SD_ERR_UNSUPPORTED, "d2sd_suffix_merge: block_len must be <= 64");
  if ((k_local == nullptr) != (v_local == nullptr))
    return fail(D2SD_ERR_INVALID_ARGUMENT, "d2sd_suffix_merge: k_local and v_local go together");
  if (k_local && !q)
    return fail(D2SD_ERR_INVALID_ARGUMENT, "d2sd_suffix_merge: q is required with k_local");
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
  SuffixParams prm;
  prm.q = q;
  prm.q_st = q_stride_token;
  prm.q_sh = q_stride_head;
  prm.k = k_local;
  prm.v = v_local;
  prm.kv_st = kv_stride_token;
  prm.kv_sh = kv_stride_head;
  prm.num_blocks = num_blocks;
  prm.block_len = block_len;
  prm.mask_mode = mask_mode;
  prm.custom_mask = custom_mask;
  prm.partial = static_cast<const float*>(partial);
  prm.plan = plan;
  prm.prefix_token = prefix_token;
  prm.prefix_out = prefix_out;
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
  prm.sink_mode = sink_mode;
  prm.Hq = num_qo_heads;
  prm.Hk = num_kv_heads;
  prm.G = num_qo_heads / num_kv_heads;
  prm.scale_log2 = sm_scale * kLog2e;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == D2SD_DTYPE_BF16) {
    return head_dim == 128 ? launch_suffix<__nv_bfloat16, 128>(prm, st)
                           : launch_suffix<__nv_bfloat16, 64>(prm, st);
  }
  if (dtype == D2SD_DTYPE_F16) {
    return head_dim == 128 ? launch_suffix<__half, 128>(prm, st) : launch_suffix<__half, 64>(prm, st);
  }
  return fail(D2SD_ERR_UNSUPPORTED, "d2sd_suffix_merge: dtype must be bf16 or f16");
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
