// Host-side planner of the shared-prefix attention (pure C++, no CUDA calls).
//
// Replaces the implicit "one FlashInfer prefill per layer over the whole
// prefix" of generation/verification.py:139-150 (and model/dflash.py:106-117)
// with an explicit partition of (request, kv head, query-tile pair, KV tile)
// work over a persistent grid, see plan_layout.h.
#include <algorithm>
#include <cstdint>
#include <cstring>
#include <string>
#include <vector>

#include "../../include/d2sd.h"
#include "plan_layout.h"

namespace d2sd {
void set_last_error(const std::string& msg);
}

using namespace d2sd::plan;

namespace {

int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

struct PairGroup {  // one (request, kv head, pair group): a run of columns
  int32_t req, head, pg;
  int64_t ntile;       // columns
  int64_t col_begin;   // first global column
  int32_t nseg = 0;    // segments (= partial slots per query tile)
};

}  // namespace

extern "C" int64_t d2sd_prefix_plan_capacity(int32_t num_requests, int32_t num_qo_heads,
                                             int32_t num_kv_heads, int32_t num_ctas,
                                             int64_t total_q_tokens) {
  if (num_requests < 0 || num_kv_heads <= 0 || num_qo_heads <= 0 || num_ctas <= 0 ||
      total_q_tokens < 0)
    return -1;
  const int64_t G = std::max<int64_t>(1, num_qo_heads / num_kv_heads);
  const int64_t R = num_requests, Hk = num_kv_heads;
  const int64_t pairs = Hk * (ceil_div(total_q_tokens * G, 2 * kTileRows) + R + 1);
  const int64_t units = Hk * (ceil_div(total_q_tokens * G, kTileRows) + R + 1);
  return kHeaderInts + (num_ctas + 1) + int64_t(kItemInts) * (num_ctas + pairs) +
         int64_t(kUnitInts) * units + int64_t(kReqInts) * R + total_q_tokens + 64;
}

extern "C" int d2sd_prefix_plan(const int32_t* q_tokens, const int32_t* q_token_offset,
                                const int32_t* kv_start, const int32_t* kv_end,
                                int32_t num_requests, int32_t num_qo_heads,
                                int32_t num_kv_heads, int32_t num_ctas, int32_t* plan,
                                int64_t capacity, int32_t* num_partial_slots) {
  using d2sd::set_last_error;
  if (num_requests < 0 || num_qo_heads <= 0 || num_kv_heads <= 0 || num_ctas <= 0 ||
      plan == nullptr || (num_requests > 0 && (!q_tokens || !q_token_offset || !kv_start ||
                                               !kv_end))) {
    set_last_error("d2sd_prefix_plan: invalid argument");
    return D2SD_ERR_INVALID_ARGUMENT;
  }
  if (num_qo_heads % num_kv_heads != 0) {
    set_last_error("d2sd_prefix_plan: num_qo_heads must be a multiple of num_kv_heads");
    return D2SD_ERR_INVALID_ARGUMENT;
  }
  const int32_t G = num_qo_heads / num_kv_heads;
  if (kTileRows % G != 0) {
    set_last_error("d2sd_prefix_plan: qo heads per kv head must divide 128");
    return D2SD_ERR_UNSUPPORTED;
  }
  const int32_t Hk = num_kv_heads;
  const int32_t R = num_requests;

  // --- per-request shapes -------------------------------------------------
  std::vector<int64_t> nqt(R), npair(R), t_lo(R), ntile(R);
  int64_t num_tokens = 0;
  for (int32_t r = 0; r < R; ++r) {
    if (q_tokens[r] < 0 || q_token_offset[r] < 0 || kv_start[r] < 0 ||
        kv_end[r] < kv_start[r]) {
      set_last_error("d2sd_prefix_plan: request " + std::to_string(r) +
                     " has a negative size or kv_end < kv_start");
      return D2SD_ERR_INVALID_ARGUMENT;
    }
    nqt[r] = ceil_div(int64_t(q_tokens[r]) * G, kTileRows);
    npair[r] = ceil_div(nqt[r], 2);
    if (kv_end[r] > kv_start[r] && q_tokens[r] > 0) {
      t_lo[r] = kv_start[r] / kTileKeys;
      ntile[r] = ceil_div(kv_end[r], kTileKeys) - t_lo[r];
    } else {
      t_lo[r] = 0;
      ntile[r] = 0;
    }
    num_tokens = std::max<int64_t>(num_tokens, int64_t(q_token_offset[r]) + q_tokens[r]);
  }

  // --- group size: CTAs that share the KV stream of one (request, head) ----
  int64_t gs = -1;
  for (int32_t r = 0; r < R; ++r) {
    if (ntile[r] == 0) continue;
    if (gs < 0) gs = npair[r];
    else if (gs != npair[r]) gs = 1;
  }
  if (gs < 1 || gs > num_ctas) gs = 1;
  const int64_t max_groups = num_ctas / gs;

  // --- pair groups (runs of columns) ---------------------------------------
  std::vector<PairGroup> pgs;
  int64_t C = 0;
  for (int32_t r = 0; r < R; ++r) {
    if (ntile[r] == 0) continue;
    const int64_t n_pg = npair[r] / gs;
    for (int32_t h = 0; h < Hk; ++h) {
      for (int64_t pg = 0; pg < n_pg; ++pg) {
        PairGroup p;
        p.req = r;
        p.head = h;
        p.pg = static_cast<int32_t>(pg);
        p.ntile = ntile[r];
        p.col_begin = C;
        C += ntile[r];
        pgs.push_back(p);
      }
    }
  }
  const int64_t NG = std::min<int64_t>(max_groups, C);  // groups actually used

  // Segments: (pair group index, first column offset, end column offset), per group.
  struct Seg {
    int64_t pgi, c0, c1, idx_in_pg;
  };
  std::vector<std::vector<Seg>> group_segs(NG);
  {
    size_t cur = 0;
    for (int64_t g = 0; g < NG; ++g) {
      const int64_t a = (C * g) / NG, b = (C * (g + 1)) / NG;
      while (cur < pgs.size() && pgs[cur].col_begin + pgs[cur].ntile <= a) ++cur;
      for (size_t u = cur; u < pgs.size() && pgs[u].col_begin < b; ++u) {
        const int64_t c0 = std::max(a, pgs[u].col_begin) - pgs[u].col_begin;
        const int64_t c1 = std::min(b, pgs[u].col_begin + pgs[u].ntile) - pgs[u].col_begin;
        if (c1 <= c0) continue;
        group_segs[g].push_back({static_cast<int64_t>(u), c0, c1, pgs[u].nseg});
        pgs[u].nseg += 1;
      }
    }
  }

  // --- units and slots -----------------------------------------------------
  std::vector<int64_t> unit_base(R);
  int64_t num_units = 0;
  for (int32_t r = 0; r < R; ++r) {
    unit_base[r] = num_units;
    num_units += int64_t(Hk) * nqt[r];
  }
  std::vector<int64_t> unit_slot_base(num_units, 0), unit_nslots(num_units, 0);
  // nslots of a unit = segments of its pair group.
  for (const PairGroup& p : pgs) {
    for (int64_t k = 0; k < gs; ++k) {
      const int64_t pair = int64_t(p.pg) * gs + k;
      for (int64_t t = 0; t < 2; ++t) {
        const int64_t qt = 2 * pair + t;
        if (qt >= nqt[p.req]) continue;
        unit_nslots[unit_base[p.req] + int64_t(p.head) * nqt[p.req] + qt] = p.nseg;
      }
    }
  }
  int64_t num_slots = 0;
  for (int64_t u = 0; u < num_units; ++u) {
    unit_slot_base[u] = num_slots;
    num_slots += unit_nslots[u];
  }

  const int64_t num_ctas_used = NG * gs;
  int64_t num_items = 0;
  for (int64_t g = 0; g < NG; ++g) num_items += int64_t(group_segs[g].size()) * gs;

  const int64_t off_cta = kHeaderInts;
  const int64_t off_items = off_cta + num_ctas_used + 1;
  const int64_t off_units = off_items + num_items * kItemInts;
  const int64_t off_req = off_units + num_units * kUnitInts;
  const int64_t off_tok = off_req + int64_t(R) * kReqInts;
  const int64_t total = off_tok + num_tokens;
  if (total > capacity) {
    set_last_error("d2sd_prefix_plan: plan needs " + std::to_string(total) +
                   " int32 entries, capacity is " + std::to_string(capacity));
    return D2SD_ERR_WORKSPACE;
  }
  if (total > INT32_MAX || num_slots > INT32_MAX) {
    set_last_error("d2sd_prefix_plan: plan too large");
    return D2SD_ERR_UNSUPPORTED;
  }

  std::memset(plan, 0, sizeof(int32_t) * kHeaderInts);
  plan[H_MAGIC] = kMagic;
  plan[H_NUM_CTAS] = static_cast<int32_t>(num_ctas_used);
  plan[H_NUM_ITEMS] = static_cast<int32_t>(num_items);
  plan[H_NUM_UNITS] = static_cast<int32_t>(num_units);
  plan[H_NUM_REQUESTS] = R;
  plan[H_NUM_SLOTS] = static_cast<int32_t>(num_slots);
  plan[H_NUM_TOKENS] = static_cast<int32_t>(num_tokens);
  plan[H_OFF_CTA] = static_cast<int32_t>(off_cta);
  plan[H_OFF_ITEMS] = static_cast<int32_t>(off_items);
  plan[H_OFF_UNITS] = static_cast<int32_t>(off_units);
  plan[H_OFF_REQUESTS] = static_cast<int32_t>(off_req);
  plan[H_OFF_TOKENS] = static_cast<int32_t>(off_tok);
  plan[H_GROUP] = G;
  plan[H_NUM_KV_HEADS] = Hk;
  plan[H_GROUP_CTAS] = static_cast<int32_t>(gs);

  // --- items, CTA by CTA (cta = group * gs + k) ----------------------------
  int64_t item = 0;
  for (int64_t g = 0; g < NG; ++g) {
    for (int64_t k = 0; k < gs; ++k) {
      plan[off_cta + g * gs + k] = static_cast<int32_t>(item);
      for (const Seg& s : group_segs[g]) {
        const PairGroup& p = pgs[s.pgi];
        const int32_t r = p.req;
        const int64_t pair = int64_t(p.pg) * gs + k;
        const int64_t qt0 = 2 * pair;
        const bool has_t1 = qt0 + 1 < nqt[r];
        const int64_t u0 = unit_base[r] + int64_t(p.head) * nqt[r] + qt0;
        int32_t* it = plan + off_items + item * kItemInts;
        it[I_REQ] = r;
        it[I_HEAD] = p.head;
        it[I_QTILE] = static_cast<int32_t>(qt0);
        it[I_HAS_T1] = has_t1 ? 1 : 0;
        it[I_T0] = static_cast<int32_t>(t_lo[r] + s.c0);
        it[I_T1] = static_cast<int32_t>(t_lo[r] + s.c1);
        it[I_KV_START] = kv_start[r];
        it[I_KV_END] = kv_end[r];
        it[I_SLOT0] = static_cast<int32_t>(unit_slot_base[u0] + s.idx_in_pg);
        it[I_SLOT1] = has_t1 ? static_cast<int32_t>(unit_slot_base[u0 + 1] + s.idx_in_pg) : -1;
        it[I_QTOK] = static_cast<int32_t>(q_token_offset[r] + qt0 * (kTileRows / G));
        it[11] = 0;
        ++item;
      }
    }
  }
  plan[off_cta + num_ctas_used] = static_cast<int32_t>(item);

  for (int64_t u = 0; u < num_units; ++u) {
    plan[off_units + u * kUnitInts + 0] = static_cast<int32_t>(unit_slot_base[u]);
    plan[off_units + u * kUnitInts + 1] = static_cast<int32_t>(unit_nslots[u]);
  }
  for (int64_t t = 0; t < num_tokens; ++t) plan[off_tok + t] = -1;
  for (int32_t r = 0; r < R; ++r) {
    int32_t* rq = plan + off_req + int64_t(r) * kReqInts;
    rq[0] = static_cast<int32_t>(unit_base[r]);
    rq[1] = static_cast<int32_t>(nqt[r]);
    rq[2] = q_token_offset[r];
    rq[3] = q_tokens[r];
    for (int32_t t = 0; t < q_tokens[r]; ++t) {
      int32_t& slot = plan[off_tok + q_token_offset[r] + t];
      if (slot != -1) {
        set_last_error("d2sd_prefix_plan: requests overlap in the Q tensor");
        return D2SD_ERR_INVALID_ARGUMENT;
      }
      slot = r;
    }
  }
  if (num_partial_slots) *num_partial_slots = static_cast<int32_t>(num_slots);
  return D2SD_OK;
}
