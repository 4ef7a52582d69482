// Kernel (d): accepted-branch KV commit for every layer in one launch.
//
// Reference (generation/d3_generator.py:227-232):
//   for each layer: cache.K = cat(cache.K, new_K[vb, :, :acc]); same for V
// which reallocates and copies the whole cache every step. Here the cache has
// fixed capacity (paged or contiguous) and only the acc accepted rows move:
// block positions 0..acc-1 of the winning branch (anchor + accepted drafts,
// not the bonus token) land at cache positions len .. len+acc-1. acc and the
// branch are read on the device from the acceptance kernel's result, so the
// host never waits between acceptance and commit.
//
// Cache formats: D2SD_KV_ROWS (rows contiguous, any page/slot/head strides) and
// D2SD_KV_UMMA_PAGES (16-key pages in the tensor core's core-matrix order).
// One 16-byte vector per thread; a row of head_dim elements is handled by
// head_dim*elem/16 consecutive threads, so each warp moves whole rows with
// fully coalesced loads and stores.
#include "common.cuh"

namespace d2sd {
namespace {

constexpr int kThreads = 256;

// The context-feature gather of d2sd_commit_kv_hidden (n == 0: none).
struct HiddenGather {
  const void* const* src;
  int n;
  int vec_per_row;  // 16-byte vectors of one source row
  int64_t s_branch, s_token;
  int elem_bytes;
  void* dst;
  int64_t d_token;
};

__global__ void __launch_bounds__(kThreads)
    commit_kernel(const void* const* __restrict__ layer_ptrs, int L, int Hk, int TB,
                  int vec_per_row, int64_t n_sb, int64_t n_sh, int64_t n_st, int64_t c_sp,
                  int64_t c_ss, int64_t c_sh, int page_size, int umma_pages,
                  const int32_t* __restrict__ page_table,
                  const int32_t* __restrict__ accept_result, const int32_t* __restrict__ len_dev,
                  int64_t len_host, int elem_bytes, HiddenGather hg) {
  const int acc = accept_result[0];
  const int branch = accept_result[1];
  const int64_t len = len_dev ? static_cast<int64_t>(*len_dev) : len_host;
  // vector id -> (layer, kv, head, t, v)
  const int64_t total = static_cast<int64_t>(L) * 2 * Hk * TB * vec_per_row;
  const int64_t total_h = static_cast<int64_t>(hg.n) * TB * hg.vec_per_row;
  for (int64_t id = blockIdx.x * static_cast<int64_t>(kThreads) + threadIdx.x; id < total + total_h;
       id += static_cast<int64_t>(gridDim.x) * kThreads) {
    if (id >= total) {
      // context feature: vector vv of row t of selected layer j
      int64_t y = id - total;
      const int vv = static_cast<int>(y % hg.vec_per_row);
      y /= hg.vec_per_row;
      const int t = static_cast<int>(y % TB);
      const int j = static_cast<int>(y / TB);
      if (t >= acc) continue;
      const uint8_t* hs = static_cast<const uint8_t*>(hg.src[j]) +
                          (branch * hg.s_branch + t * hg.s_token) * hg.elem_bytes + vv * 16;
      uint8_t* hd = static_cast<uint8_t*>(hg.dst) + t * hg.d_token * hg.elem_bytes +
                    (static_cast<int64_t>(j) * hg.vec_per_row + vv) * 16;
      *reinterpret_cast<uint4*>(hd) = *reinterpret_cast<const uint4*>(hs);
      continue;
    }
    int64_t x = id;
    const int vv = static_cast<int>(x % vec_per_row);
    x /= vec_per_row;
    const int t = static_cast<int>(x % TB);
    x /= TB;
    const int h = static_cast<int>(x % Hk);
    x /= Hk;
    const int kv = static_cast<int>(x % 2);
    const int l = static_cast<int>(x / 2);
    if (t >= acc) continue;
    const uint8_t* src = static_cast<const uint8_t*>(layer_ptrs[4 * l + kv]);
    uint8_t* dst = static_cast<uint8_t*>(const_cast<void*>(layer_ptrs[4 * l + 2 + kv]));
    const int64_t s_off = (branch * n_sb + h * n_sh + t * n_st) * elem_bytes + vv * 16;
    const int64_t pos = len + t;
    const int64_t pidx = pos / page_size;
    const int64_t page = page_table ? static_cast<int64_t>(page_table[pidx]) : pidx;
    const int r = static_cast<int>(pos % page_size);
    // UMMA pages: 16-byte chunk vv of row r sits in core matrix (r/8, vv), row r%8
    const int64_t in_page = umma_pages
                                ? ((static_cast<int64_t>(r / 8) * vec_per_row + vv) * 64 + (r % 8) * 8)
                                : static_cast<int64_t>(r) * c_ss;
    const int64_t d_off = (page * c_sp + h * c_sh + in_page) * elem_bytes + (umma_pages ? 0 : vv * 16);
    *reinterpret_cast<uint4*>(dst + d_off) = *reinterpret_cast<const uint4*>(src + s_off);
  }
}

}  // namespace
}  // namespace d2sd

namespace d2sd {
namespace {
int commit_impl(const void* const* layer_ptrs, int32_t num_layers, int32_t num_kv_heads,
                int32_t head_dim, int32_t elem_bytes, int32_t block_len, int64_t new_stride_branch,
                int64_t new_stride_head, int64_t new_stride_token, int64_t cache_stride_page,
                int64_t cache_stride_slot, int64_t cache_stride_head, int32_t page_size,
                int32_t cache_format, const int32_t* page_table, const int32_t* accept_result,
                const int32_t* cache_len_dev, int64_t cache_len_host, const HiddenGather& hg,
                void* stream) {
  if (!layer_ptrs || !accept_result || num_layers <= 0 || num_kv_heads <= 0 || head_dim <= 0 ||
      block_len <= 0 || page_size <= 0 || cache_len_host < 0)
    return fail(D2SD_ERR_INVALID_ARGUMENT, "d2sd_commit_kv: invalid argument");
  if (elem_bytes != 2 && elem_bytes != 4)
    return fail(D2SD_ERR_UNSUPPORTED, "d2sd_commit_kv: elem_bytes must be 2 or 4");
  if (cache_format != D2SD_KV_ROWS && cache_format != D2SD_KV_UMMA_PAGES)
    return fail(D2SD_ERR_INVALID_ARGUMENT, "d2sd_commit_kv: unknown cache_format");
  if (cache_format == D2SD_KV_UMMA_PAGES && (elem_bytes != 2 || page_size != 16))
    return fail(D2SD_ERR_UNSUPPORTED, "d2sd_commit_kv: UMMA pages hold 16-bit values, 16 per page");
  if ((static_cast<int64_t>(head_dim) * elem_bytes) % 16 != 0)
    return fail(D2SD_ERR_UNSUPPORTED, "d2sd_commit_kv: head_dim*elem_bytes must be a multiple of 16");
  const int64_t vec_elems = 16 / elem_bytes;
  if (new_stride_branch % vec_elems || new_stride_head % vec_elems ||
      new_stride_token % vec_elems || cache_stride_page % vec_elems ||
      cache_stride_slot % vec_elems || cache_stride_head % vec_elems)
    return fail(D2SD_ERR_INVALID_ARGUMENT, "d2sd_commit_kv: strides must keep rows 16-byte aligned");
  const int vec_per_row = head_dim * elem_bytes / 16;
  const int64_t total = static_cast<int64_t>(num_layers) * 2 * num_kv_heads * block_len * vec_per_row +
                        static_cast<int64_t>(hg.n) * block_len * hg.vec_per_row;
  int64_t blocks = (total + kThreads - 1) / kThreads;
  const int64_t max_blocks = static_cast<int64_t>(current_sm_count()) * 16;
  if (blocks > max_blocks) blocks = max_blocks;
  commit_kernel<<<static_cast<unsigned>(blocks), kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      layer_ptrs, num_layers, num_kv_heads, block_len, vec_per_row, new_stride_branch,
      new_stride_head, new_stride_token, cache_stride_page, cache_stride_slot, cache_stride_head,
      page_size, cache_format == D2SD_KV_UMMA_PAGES ? 1 : 0, page_table, accept_result,
      cache_len_dev, cache_len_host, elem_bytes, hg);
  return check_launch("commit_kernel");
}
}  // namespace
}  // namespace d2sd

extern "C" int d2sd_commit_kv(const void* const* layer_ptrs, int32_t num_layers,
                              int32_t num_kv_heads, int32_t head_dim, int32_t elem_bytes,
                              int32_t block_len, int64_t new_stride_branch,
                              int64_t new_stride_head, int64_t new_stride_token,
                              int64_t cache_stride_page, int64_t cache_stride_slot,
                              int64_t cache_stride_head, int32_t page_size, int32_t cache_format,
                              const int32_t* page_table, const int32_t* accept_result,
                              const int32_t* cache_len_dev, int64_t cache_len_host, void* stream) {
  d2sd::HiddenGather none{};
  return d2sd::commit_impl(layer_ptrs, num_layers, num_kv_heads, head_dim, elem_bytes, block_len,
                           new_stride_branch, new_stride_head, new_stride_token,
                           cache_stride_page, cache_stride_slot, cache_stride_head, page_size,
                           cache_format, page_table, accept_result, cache_len_dev,
                           cache_len_host, none, stream);
}

extern "C" int d2sd_commit_kv_hidden(
    const void* const* layer_ptrs, int32_t num_layers, int32_t num_kv_heads, int32_t head_dim,
    int32_t elem_bytes, int32_t block_len, int64_t new_stride_branch, int64_t new_stride_head,
    int64_t new_stride_token, int64_t cache_stride_page, int64_t cache_stride_slot,
    int64_t cache_stride_head, int32_t page_size, int32_t cache_format, const int32_t* page_table,
    const int32_t* accept_result, const int32_t* cache_len_dev, int64_t cache_len_host,
    const void* const* hidden_src, int32_t num_hidden, int32_t hidden_size,
    int32_t hidden_elem_bytes, int64_t hidden_stride_branch, int64_t hidden_stride_token,
    void* hidden_dst, int64_t hidden_dst_stride_token, void* stream) {
  using namespace d2sd;
  if (num_hidden < 0 || (num_hidden > 0 && (!hidden_src || !hidden_dst || hidden_size <= 0)))
    return fail(D2SD_ERR_INVALID_ARGUMENT, "d2sd_commit_kv_hidden: invalid hidden argument");
  if (hidden_elem_bytes != 2 && hidden_elem_bytes != 4)
    return fail(D2SD_ERR_UNSUPPORTED, "d2sd_commit_kv_hidden: hidden_elem_bytes must be 2 or 4");
  const int64_t ve = 16 / hidden_elem_bytes;
  if (hidden_size % ve || hidden_stride_branch % ve || hidden_stride_token % ve ||
      hidden_dst_stride_token % ve || (num_hidden > 0 && !aligned16(hidden_dst)) ||
      hidden_dst_stride_token < static_cast<int64_t>(num_hidden) * hidden_size)
    return fail(D2SD_ERR_INVALID_ARGUMENT,
                "d2sd_commit_kv_hidden: hidden rows must be 16-byte aligned and the destination "
                "rows at least num_hidden*hidden_size wide");
  HiddenGather hg;
  hg.src = hidden_src;
  hg.n = num_hidden;
  hg.vec_per_row = static_cast<int>(hidden_size / ve);
  hg.s_branch = hidden_stride_branch;
  hg.s_token = hidden_stride_token;
  hg.elem_bytes = hidden_elem_bytes;
  hg.dst = hidden_dst;
  hg.d_token = hidden_dst_stride_token;
  return commit_impl(layer_ptrs, num_layers, num_kv_heads, head_dim, elem_bytes, block_len,
                     new_stride_branch, new_stride_head, new_stride_token, cache_stride_page,
                     cache_stride_slot, cache_stride_head, page_size, cache_format, page_table,
                     accept_result, cache_len_dev, cache_len_host, hg, stream);
}
