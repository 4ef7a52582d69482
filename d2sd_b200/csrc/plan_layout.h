// Layout of the int32 work plan shared by the host planner (plan.cpp), the
// shared-prefix attention kernel (prefix_attn.cu) and the merge kernel
// (suffix_merge.cu).
//
// The prefix attention is a persistent kernel. Its unit of work is a "column":
// one 128-key KV tile of one (request, kv head) against a pair of 128-row query
// tiles (rows are token*G + g for the G query heads of that kv head). CTAs are
// arranged in groups of `group_ctas`; the CTAs of a group take consecutive query
// tile pairs of the same (request, kv head) and walk the SAME contiguous range
// of columns, so each KV tile is fetched from HBM once per group and served to
// the other CTAs of the group from L2. Each CTA's column range is cut into
// items at (request, kv head) boundaries; every item writes one partial state
// (normalised O and base-2 LSE per row) per query tile into a "slot", and the
// slots of a query tile are merged later by the suffix/merge kernel.
#pragma once

#include <stdint.h>

#ifdef __CUDACC__
#define D2SD_HOST_DEVICE __host__ __device__
#else
#define D2SD_HOST_DEVICE
#endif

namespace d2sd {
namespace plan {

constexpr int32_t kMagic = 0x44325344;  // "D2SD"
constexpr int kTileKeys = 128;          // keys per KV tile (UMMA N of Q.K^T)
constexpr int kTileRows = 128;          // query rows per tile (TMEM lanes)

// header
constexpr int kHeaderInts = 16;
constexpr int H_MAGIC = 0;
constexpr int H_NUM_CTAS = 1;      // CTAs the prefix kernel is launched with
constexpr int H_NUM_ITEMS = 2;
constexpr int H_NUM_UNITS = 3;     // (request, kv head, query tile) triples
constexpr int H_NUM_REQUESTS = 4;
constexpr int H_NUM_SLOTS = 5;     // partial-state slots written
constexpr int H_NUM_TOKENS = 6;    // rows of the token -> request table
constexpr int H_OFF_CTA = 7;       // cta item offsets [num_ctas + 1]
constexpr int H_OFF_ITEMS = 8;     // items [num_items][kItemInts]
constexpr int H_OFF_UNITS = 9;     // units [num_units][kUnitInts]
constexpr int H_OFF_REQUESTS = 10; // requests [num_requests][kReqInts]
constexpr int H_OFF_TOKENS = 11;   // token -> request [num_tokens]
constexpr int H_GROUP = 12;        // G = qo heads per kv head
constexpr int H_NUM_KV_HEADS = 13;
constexpr int H_GROUP_CTAS = 14;   // CTAs per group

// item
constexpr int kItemInts = 12;
constexpr int I_REQ = 0;
constexpr int I_HEAD = 1;       // kv head
constexpr int I_QTILE = 2;      // first query tile of the pair
constexpr int I_HAS_T1 = 3;     // second query tile exists
constexpr int I_T0 = 4;         // first KV tile (absolute, in 128-key units)
constexpr int I_T1 = 5;         // one past the last KV tile
constexpr int I_KV_START = 6;   // first visible key position
constexpr int I_KV_END = 7;     // one past the last visible key position
constexpr int I_SLOT0 = 8;      // partial slot of query tile 0
constexpr int I_SLOT1 = 9;      // partial slot of query tile 1 (-1 if none)
constexpr int I_QTOK = 10;      // Q-tensor token index of query tile 0's row 0

// Partial-state slot (one per item per query tile): the normalised O of its
// 128 rows in bf16 ([128][head_dim], row-major), then their base-2 LSEs in fp32.
D2SD_HOST_DEVICE constexpr int64_t slot_bytes(int head_dim) {
  return static_cast<int64_t>(kTileRows) * head_dim * 2 + kTileRows * 4;
}

// unit: (slot_base, num_slots)
constexpr int kUnitInts = 2;
// request: (unit_base, num_query_tiles, q_token_offset, q_tokens)
constexpr int kReqInts = 4;

}  // namespace plan
}  // namespace d2sd
