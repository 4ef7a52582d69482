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
// A thread owns one 16-byte vector position (request, layer, K|V, head, chunk)
// and moves that chunk for every accepted position t < acc, the loads of up to
// four positions in flight before their stores; consecutive threads take
// consecutive chunks of a row, so a warp moves whole rows coalesced. acc, the
// branch and the cache length are read once per thread from the acceptance
// result, and no thread is spent on rejected positions.
// The batched form (d2sd_commit_kv_batch) adds the request dimension for
// batched serving: per request its own acceptance result, cache length and
// page-table offset, all requests' caches in one pool per layer.
#include "common.cuh"

namespace d2sd {
namespace {

constexpr int kThreads = 256;
constexpr int kUnroll = 4;

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

struct CommitArgs {
  const void* const* layer_ptrs;  // [L][4] {new_k, new_v, cache_k, cache_v}
  int R, L, Hk, TB, vec_per_row, elem_bytes;
  int64_t n_sr, n_sb, n_sh, n_st;  // new K/V element strides (request, branch, head, token)
  int64_t c_sp, c_ss, c_sh;        // cache element strides (page, slot, head)
  int page_size, umma_pages;
  const int32_t* page_table;
  const int32_t* page_table_offset;  // [R] or NULL
  const int32_t* accept_result;      // [R][2] {acc, branch}
  const int32_t* len_dev;            // [R] or NULL
  int64_t len_host;                  // cache length when len_dev is NULL (R == 1)
};

__global__ void __launch_bounds__(kThreads)
    commit_kernel(const CommitArgs a, const HiddenGather hg) {
  // launched with programmatic serialisation: everything below reads the
  // acceptance result of the previous kernel
  grid_dep_wait();
  const int64_t per_req = static_cast<int64_t>(a.L) * 2 * a.Hk * a.vec_per_row;
  const int64_t total = per_req * a.R;
  const int64_t total_h = static_cast<int64_t>(hg.n) * hg.vec_per_row;
  for (int64_t id = blockIdx.x * static_cast<int64_t>(kThreads) + threadIdx.x; id < total + total_h;
       id += static_cast<int64_t>(gridDim.x) * kThreads) {
    if (id >= total) {
      // context feature (one request): chunk vv of selected layer j, rows t < acc
      const int64_t y = id - total;
      const int vv = static_cast<int>(y % hg.vec_per_row);
      const int j = static_cast<int>(y / hg.vec_per_row);
      const int acc = min(max(a.accept_result[0], 0), a.TB), branch = a.accept_result[1];
      const uint8_t* hs = static_cast<const uint8_t*>(hg.src[j]) +
                          branch * hg.s_branch * hg.elem_bytes + vv * 16;
      uint8_t* hd = static_cast<uint8_t*>(hg.dst) +
                    (static_cast<int64_t>(j) * hg.vec_per_row + vv) * 16;
      for (int t0 = 0; t0 < acc; t0 += kUnroll) {
        uint4 v[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u)
          if (t0 + u < acc)
            v[u] = *reinterpret_cast<const uint4*>(hs + (t0 + u) * hg.s_token * hg.elem_bytes);
#pragma unroll
        for (int u = 0; u < kUnroll; ++u)
          if (t0 + u < acc)
            *reinterpret_cast<uint4*>(hd + (t0 + u) * hg.d_token * hg.elem_bytes) = v[u];
      }
      continue;
    }
    int64_t x = id;
    const int vv = static_cast<int>(x % a.vec_per_row);
    x /= a.vec_per_row;
    const int h = static_cast<int>(x % a.Hk);
    x /= a.Hk;
    const int kv = static_cast<int>(x % 2);
    x /= 2;
    const int l = static_cast<int>(x % a.L);
    const int r = static_cast<int>(x / a.L);
    const int acc = min(max(a.accept_result[2 * r], 0), a.TB);  // never past the block
    const int branch = a.accept_result[2 * r + 1];
    const int64_t len = a.len_dev ? static_cast<int64_t>(a.len_dev[r]) : a.len_host;
    const int32_t* pt = a.page_table ? a.page_table + (a.page_table_offset ? a.page_table_offset[r] : 0)
                                     : nullptr;
    const uint8_t* src = static_cast<const uint8_t*>(a.layer_ptrs[4 * l + kv]) +
                         ((r * a.n_sr + branch * a.n_sb + h * a.n_sh) * a.elem_bytes + vv * 16);
    uint8_t* dst = static_cast<uint8_t*>(const_cast<void*>(a.layer_ptrs[4 * l + 2 + kv]));
    for (int t0 = 0; t0 < acc; t0 += kUnroll) {
      // the rows and their pages are loaded before any store (a store through
      // the byte pointer could alias a later load and would serialise them)
      uint4 v[kUnroll];
      int64_t page[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        if (t0 + u < acc) {
          v[u] = __ldg(reinterpret_cast<const uint4*>(src + (t0 + u) * a.n_st * a.elem_bytes));
          const int64_t pidx = (len + t0 + u) / a.page_size;
          page[u] = pt ? static_cast<int64_t>(__ldg(pt + pidx)) : pidx;
        }
      }
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        if (t0 + u >= acc) break;
        const int64_t pos = len + t0 + u;
        const int s = static_cast<int>(pos % a.page_size);
        // UMMA pages: 16-byte chunk vv of row s sits in core matrix (s/8, vv), row s%8
        const int64_t in_page =
            a.umma_pages ? ((static_cast<int64_t>(s / 8) * a.vec_per_row + vv) * 64 + (s % 8) * 8)
                         : static_cast<int64_t>(s) * a.c_ss;
        const int64_t d_off =
            (page[u] * a.c_sp + h * a.c_sh + in_page) * a.elem_bytes + (a.umma_pages ? 0 : vv * 16);
        *reinterpret_cast<uint4*>(dst + d_off) = v[u];
      }
    }
  }
}

}  // namespace
}  // namespace d2sd

namespace d2sd {
namespace {
int commit_impl(CommitArgs a, int32_t head_dim, int32_t cache_format, const HiddenGather& hg,
                void* stream, const char* what) {
  const std::string w(what);
  if (!a.layer_ptrs || !a.accept_result || a.R <= 0 || a.L <= 0 || a.Hk <= 0 || head_dim <= 0 ||
      a.TB <= 0 || a.page_size <= 0 || a.len_host < 0)
    return fail(D2SD_ERR_INVALID_ARGUMENT, w + ": invalid argument");
  if (a.elem_bytes != 2 && a.elem_bytes != 4)
    return fail(D2SD_ERR_UNSUPPORTED, w + ": elem_bytes must be 2 or 4");
  if (cache_format != D2SD_KV_ROWS && cache_format != D2SD_KV_UMMA_PAGES)
    return fail(D2SD_ERR_INVALID_ARGUMENT, w + ": unknown cache_format");
  if (cache_format == D2SD_KV_UMMA_PAGES && (a.elem_bytes != 2 || a.page_size != 16))
    return fail(D2SD_ERR_UNSUPPORTED, w + ": UMMA pages hold 16-bit values, 16 per page");
  if ((static_cast<int64_t>(head_dim) * a.elem_bytes) % 16 != 0)
    return fail(D2SD_ERR_UNSUPPORTED, w + ": head_dim*elem_bytes must be a multiple of 16");
  const int64_t vec_elems = 16 / a.elem_bytes;
  if (a.n_sr % vec_elems || a.n_sb % vec_elems || a.n_sh % vec_elems || a.n_st % vec_elems ||
      a.c_sp % vec_elems || a.c_ss % vec_elems || a.c_sh % vec_elems)
    return fail(D2SD_ERR_INVALID_ARGUMENT, w + ": strides must keep rows 16-byte aligned");
  a.vec_per_row = head_dim * a.elem_bytes / 16;
  a.umma_pages = cache_format == D2SD_KV_UMMA_PAGES ? 1 : 0;
  const int64_t total = static_cast<int64_t>(a.R) * a.L * 2 * a.Hk * a.vec_per_row +
                        static_cast<int64_t>(hg.n) * hg.vec_per_row;
  int64_t blocks = (total + kThreads - 1) / kThreads;
  const int64_t max_blocks = static_cast<int64_t>(current_sm_count()) * 8;
  if (blocks > max_blocks) blocks = max_blocks;
  return launch_pdl(commit_kernel, dim3(static_cast<unsigned>(blocks)), dim3(kThreads), 0,
                    static_cast<cudaStream_t>(stream), "commit_kernel", a, hg);
}

CommitArgs single_args(const void* const* layer_ptrs, int32_t num_layers, int32_t num_kv_heads,
                       int32_t elem_bytes, int32_t block_len, int64_t nsb, int64_t nsh,
                       int64_t nst, int64_t csp, int64_t css, int64_t csh, int32_t page_size,
                       const int32_t* page_table, const int32_t* accept_result,
                       const int32_t* cache_len_dev, int64_t cache_len_host) {
  CommitArgs a{};
  a.layer_ptrs = layer_ptrs;
  a.R = 1;
  a.L = num_layers;
  a.Hk = num_kv_heads;
  a.TB = block_len;
  a.elem_bytes = elem_bytes;
  a.n_sr = 0;
  a.n_sb = nsb;
  a.n_sh = nsh;
  a.n_st = nst;
  a.c_sp = csp;
  a.c_ss = css;
  a.c_sh = csh;
  a.page_size = page_size;
  a.page_table = page_table;
  a.page_table_offset = nullptr;
  a.accept_result = accept_result;
  a.len_dev = cache_len_dev;
  a.len_host = cache_len_host;
  return a;
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
  using namespace d2sd;
  const CommitArgs a = single_args(layer_ptrs, num_layers, num_kv_heads, elem_bytes, block_len,
                                   new_stride_branch, new_stride_head, new_stride_token,
                                   cache_stride_page, cache_stride_slot, cache_stride_head,
                                   page_size, page_table, accept_result, cache_len_dev,
                                   cache_len_host);
  return commit_impl(a, head_dim, cache_format, HiddenGather{}, stream, "d2sd_commit_kv");
}

extern "C" int d2sd_commit_kv_batch(const void* const* layer_ptrs, int32_t num_layers,
                                    int32_t num_requests, int32_t num_kv_heads, int32_t head_dim,
                                    int32_t elem_bytes, int32_t block_len,
                                    int64_t new_stride_request, int64_t new_stride_branch,
                                    int64_t new_stride_head, int64_t new_stride_token,
                                    int64_t cache_stride_page, int64_t cache_stride_slot,
                                    int64_t cache_stride_head, int32_t page_size,
                                    int32_t cache_format, const int32_t* page_table,
                                    const int32_t* page_table_offset,
                                    const int32_t* accept_results, const int32_t* cache_lens,
                                    void* stream) {
  using namespace d2sd;
  if (!cache_lens || !page_table || !page_table_offset)
    return fail(D2SD_ERR_INVALID_ARGUMENT,
                "d2sd_commit_kv_batch: cache lengths, page table and page-table offsets are required");
  CommitArgs a = single_args(layer_ptrs, num_layers, num_kv_heads, elem_bytes, block_len,
                             new_stride_branch, new_stride_head, new_stride_token,
                             cache_stride_page, cache_stride_slot, cache_stride_head, page_size,
                             page_table, accept_results, cache_lens, 0);
  a.R = num_requests;
  a.n_sr = new_stride_request;
  a.page_table_offset = page_table_offset;
  return commit_impl(a, head_dim, cache_format, HiddenGather{}, stream, "d2sd_commit_kv_batch");
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
  const CommitArgs a = single_args(layer_ptrs, num_layers, num_kv_heads, elem_bytes, block_len,
                                   new_stride_branch, new_stride_head, new_stride_token,
                                   cache_stride_page, cache_stride_slot, cache_stride_head,
                                   page_size, page_table, accept_result, cache_len_dev,
                                   cache_len_host);
  return commit_impl(a, head_dim, cache_format, hg, stream, "d2sd_commit_kv_hidden");
}
