// Compiled block-mask plan: layout shared by the plan compiler and the attention kernels.
//
// A plan is one caller-owned device buffer of int32 words:
//   header    kPlanHeaderWords words (magic, dims, device-written counts, forward pairing)
//   mask      raw uint8 mask [Bm, Hm, nq, nk] (copy of the caller's mask)
//   qempty    uint8 [Bm, Hm, nq]: 1 when every token of the q-block is fully masked
//   usel      uint8 [B * H]: 1 for the (b, h) units this plan computes (all by default; a rank
//             of a job sharded over GPUs selects its own units)
//   row_act   [Bm * Hm * nq]   active kv blocks of each q-block row after the causal cut
//   sel       [B * H]          selected units, ascending unit id b * H + h
//   grp_sel   [B * H]          selected units grouped by mask group, ascending within a group
//   grp_off   [Bm * Hm + 1]    start of each group in grp_sel
//   grp_poff  [Bm * Hm + 1]    start of each group's unit pairs (pairs of consecutive grp_sel)
//   -- built only when block_size % 64 == 0 and S % 64 == 0 (the tensor-core path) --
//   f_rowptr  [nrows + 1]       forward pair rows: (group g = bm*Hm + hm, pair t) covers the
//   f_entries [nrows * n64]     128 query rows of 64-token chunks 2t, 2t+1; each entry is a
//                               64-token kv chunk with per-half activity / diagonal flags
//   f_items   [B * H * npairs]  items (b*H + h)*npairs + t of the selected units, longest
//                               first (the backward's dQ pass); count in H_F_ITEMS
//   b_rowptr  [nrows + 1]       backward kv-pair columns: (g, u) covers kv chunks 2u, 2u+1;
//   b_entries [nrows * n64]     each entry is a 64-token q chunk with per-half flags
//   b_items   [B * H * npairs]  backward work items of the selected units, longest first
//                               (count in H_B_ITEMS)
//   jcnt      [Bm * Hm * n64]   steps of 64-row query chunk j: entries of row (g, j / 2) that
//                               half j % 2 attends
//   f_work    [max_work][8]     forward work table (FWork), longest first; count in H_F_WORK
//   f_tmp     [max_work][8]     scratch of the plan compiler (unsorted work table)
//   f_cost    [max_work]        scratch: steps of each unsorted entry
//   f_order   [max_work]        scratch: sorted order
#pragma once

#include <stdint.h>

namespace xsake {

constexpr int32_t kPlanMagic = 0x504B5358;  // "XSKP"
constexpr int32_t kPlanVersion = 4;
constexpr int kPlanHeaderWords = 32;

// Entry encoding: low 20 bits = chunk index, then flags.
constexpr int32_t kEntryIdxMask = (1 << 20) - 1;
constexpr int32_t kFlagActive0 = 1 << 20;  // half 0 (first 64 rows of the tile) attends
constexpr int32_t kFlagActive1 = 1 << 21;  // half 1 attends
constexpr int32_t kFlagDiag0 = 1 << 22;    // half 0 needs the token-level causal test
constexpr int32_t kFlagDiag1 = 1 << 23;    // half 1 needs the token-level causal test
constexpr int32_t kEntryFlags = 0xF << 20;  // any of the four flags

// Split pieces of the forward: a work item whose kv walk is long next to the average load
// of a worker is cut into pieces over its kv chunks; each piece writes an unnormalised
// partial (O, running max, row sum) into one slot of the forward workspace, and the piece
// that finishes last merges the slots in piece order (deterministic).
constexpr int kSplitSlots = 512;            // partial slots in the forward workspace
constexpr int kMaxPieces = 64;              // pieces of one item at most
constexpr int kMinPieceSteps = 4;           // smallest piece (kv chunks)

// Forward pairings (header word H_FWD_PAIR): which rows a work item of the tensor-core forward
// covers; every step is one 64-key chunk.
constexpr int32_t kPairQuery = 0;   // query chunks 2t, 2t+1 of one unit
constexpr int32_t kPairUnits = 1;   // query chunk j of two units that share the mask

// Forward work table entry (8 int32 words).
struct FWork {
  int32_t u0;      // unit b * H + h (query-chunk pairing: the unit; unit pairing: unit of lanes 0-15)
  int32_t u1;      // unit pairing: unit of lanes 16-31, -1 when the unit runs alone; else -1
  int32_t q;       // query-chunk pairing: 128-row tile t; unit pairing: 64-row chunk j
  int32_t lo, hi;  // range of f_entries (absolute positions) this piece walks
  int32_t parts;   // (piece index << 8) | number of pieces (1: not split)
  int32_t grp;     // split group (merge counter index), -1 when not split
  int32_t slot;    // first partial slot of the split group
};

// Header word indices.
enum PlanHeader : int {
  H_MAGIC = 0, H_VERSION, H_B, H_H, H_S, H_BM, H_HM, H_BS, H_CAUSAL, H_HAS_CSR,
  H_F_NNZ, H_B_NNZ,
  H_SEL_UNITS,      // selected units
  H_F_ITEMS,        // f_items entries
  H_B_ITEMS,        // b_items entries
  H_F_WORK,         // f_work entries
  H_ACTIVE_LO, H_ACTIVE_HI, H_TILES_LO, H_TILES_HI, H_EMPTY_LO, H_EMPTY_HI,
  H_ITEMS_LO, H_ITEMS_HI,
  H_FWD_PAIR,       // forward pairing (kPairQuery or kPairUnits; see attn_fwd_tc.cu)
  H_SPLIT_GROUPS,   // split work items
  H_SPLIT_SLOTS,    // partial slots they use
  H_SPLIT_CAP,      // largest piece (kv chunks) the split rule allowed
  H_WORKERS,        // concurrent tile workers the split rule assumed
};

__host__ __device__ __forceinline__ int32_t plan_pair_units(int32_t B, int32_t H, int32_t Bm, int32_t Hm) {
  return (Bm == 1 ? B : 1) * (Hm == 1 ? H : 1);
}

struct PlanLayout {
  int32_t B, H, S, Bm, Hm, bs, causal;
  int32_t nq, n64, npairs, nrows, nitems, has_csr, ngroups, max_work;
  int64_t mask_off, qempty_off, usel_off, row_act_off, sel_off, grp_sel_off, grp_off_off, grp_poff_off;
  int64_t f_rowptr_off, f_entries_off, f_items_off;
  int64_t b_rowptr_off, b_entries_off, b_items_off;
  int64_t jcnt_off, f_work_off, f_tmp_off, f_cost_off, f_order_off;
  int64_t total_words;

  // Returns false when the dims are invalid.
  __host__ __device__ bool init(int32_t B_, int32_t H_, int32_t S_, int32_t Bm_, int32_t Hm_,
                                int32_t bs_, int32_t causal_) {
    B = B_; H = H_; S = S_; Bm = Bm_; Hm = Hm_; bs = bs_; causal = causal_ ? 1 : 0;
    if (B <= 0 || H <= 0 || S <= 0 || bs <= 0 || S % bs) return false;
    if (!(Bm == 1 || Bm == B) || !(Hm == 1 || Hm == H)) return false;
    nq = S / bs;
    has_csr = (bs % 64 == 0 && S % 64 == 0) ? 1 : 0;
    n64 = (S + 63) / 64;
    npairs = (n64 + 1) / 2;
    ngroups = Bm * Hm;
    nrows = ngroups * npairs;
    nitems = B * H * npairs;
    const int64_t pair_max = (int64_t)n64 * ngroups * ((plan_pair_units(B, H, Bm, Hm) + 1) / 2);
    const int64_t base_max = nitems > pair_max ? nitems : pair_max;
    max_work = (int32_t)(base_max + kSplitSlots);
    int64_t w = kPlanHeaderWords;
    const int64_t mask_bytes = (int64_t)ngroups * nq * nq;
    mask_off = w;
    w += (mask_bytes + 3) / 4;
    qempty_off = w;
    w += ((int64_t)ngroups * nq + 3) / 4;
    usel_off = w;
    w += ((int64_t)B * H + 3) / 4;
    row_act_off = w;  w += (int64_t)ngroups * nq;
    sel_off = w;      w += (int64_t)B * H;
    grp_sel_off = w;  w += (int64_t)B * H;
    grp_off_off = w;  w += ngroups + 1;
    grp_poff_off = w; w += ngroups + 1;
    const int64_t csr = has_csr ? 1 : 0;
    f_rowptr_off = w;  w += csr * (nrows + 1);
    f_entries_off = w; w += csr * (int64_t)nrows * n64;
    f_items_off = w;   w += csr * nitems;
    b_rowptr_off = w;  w += csr * (nrows + 1);
    b_entries_off = w; w += csr * (int64_t)nrows * n64;
    b_items_off = w;   w += csr * nitems;
    jcnt_off = w;      w += csr * (int64_t)ngroups * n64;
    w = (w + 3) & ~(int64_t)3;   // 16-byte aligned work table
    f_work_off = w;    w += csr * (int64_t)max_work * 8;
    f_tmp_off = w;     w += csr * (int64_t)max_work * 8;
    f_cost_off = w;    w += csr * (int64_t)max_work;
    f_order_off = w;   w += csr * (int64_t)max_work;
    total_words = w;
    return true;
  }
  __host__ __device__ int32_t group_of(int32_t b, int32_t h) const {
    return (Bm == 1 ? 0 : b) * Hm + (Hm == 1 ? 0 : h);
  }
};

// True when the plan computes unit (b, h).
__device__ __forceinline__ bool plan_unit_selected(const int32_t* plan, const PlanLayout& L, int b, int h) {
  return reinterpret_cast<const uint8_t*>(plan + L.usel_off)[b * L.H + h] != 0;
}

}  // namespace xsake
