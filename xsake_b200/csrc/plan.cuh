// Compiled block-mask plan: layout shared by the plan compiler and the attention kernels.
//
// A plan is one caller-owned device buffer of int32 words:
//   header    kPlanHeaderWords words (magic, dims, device-written counts, forward pairing)
//   mask      raw uint8 mask [Bm, Hm, nq, nk] (copy of the caller's mask)
//   qempty    uint8 [Bm, Hm, nq]: 1 when every token of the q-block is fully masked
//   -- built only when block_size % 64 == 0 and S % 64 == 0 (the tensor-core path) --
//   f_rowptr  [nrows + 1]       forward pair rows: (group g = bm*Hm + hm, pair t) covers the
//   f_entries [nrows * n64]     128 query rows of 64-token chunks 2t, 2t+1; each entry is a
//                               64-token kv chunk with per-half activity / diagonal flags
//   f_items   [B * H * npairs]  forward work items (b*H + h)*npairs + t, longest first
//   b_rowptr  [nrows + 1]       backward kv-pair columns: (g, u) covers kv chunks 2u, 2u+1;
//   b_entries [nrows * n64]     each entry is a 64-token q chunk with per-half flags
//   b_items   [B * H * npairs]  backward work items, longest first
#pragma once

#include <stdint.h>

namespace xsake {

constexpr int32_t kPlanMagic = 0x504B5358;  // "XSKP"
constexpr int32_t kPlanVersion = 3;
constexpr int kPlanHeaderWords = 32;

// Entry encoding: low 20 bits = chunk index, then flags.
constexpr int32_t kEntryIdxMask = (1 << 20) - 1;
constexpr int32_t kFlagActive0 = 1 << 20;  // half 0 (first 64 rows of the tile) attends
constexpr int32_t kFlagActive1 = 1 << 21;  // half 1 attends
constexpr int32_t kFlagDiag0 = 1 << 22;    // half 0 needs the token-level causal test
constexpr int32_t kFlagDiag1 = 1 << 23;    // half 1 needs the token-level causal test
constexpr int32_t kEntryFlags = 0xF << 20;  // any of the four flags

// Header word indices.
enum PlanHeader : int {
  H_MAGIC = 0, H_VERSION, H_B, H_H, H_S, H_BM, H_HM, H_BS, H_CAUSAL, H_HAS_CSR,
  H_F_NNZ, H_B_NNZ,
  H_ACTIVE_LO = 16, H_ACTIVE_HI, H_TILES_LO, H_TILES_HI, H_EMPTY_LO, H_EMPTY_HI,
  H_ITEMS_LO, H_ITEMS_HI,
  H_FWD_PAIR,   // 1: the forward pairs units that share a mask (see attn_fwd_tc.cu), 0: query chunks
};

struct PlanLayout {
  int32_t B, H, S, Bm, Hm, bs, causal;
  int32_t nq, n64, npairs, nrows, nitems, has_csr;
  int64_t mask_off, qempty_off, f_rowptr_off, f_entries_off, f_items_off;
  int64_t b_rowptr_off, b_entries_off, b_items_off;
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
    nrows = Bm * Hm * npairs;
    nitems = B * H * npairs;
    int64_t w = kPlanHeaderWords;
    const int64_t mask_bytes = (int64_t)Bm * Hm * nq * nq;
    mask_off = w;
    w += (mask_bytes + 3) / 4;
    qempty_off = w;
    w += ((int64_t)Bm * Hm * nq + 3) / 4;
    const int64_t csr = has_csr ? 1 : 0;
    f_rowptr_off = w;  w += csr * (nrows + 1);
    f_entries_off = w; w += csr * (int64_t)nrows * n64;
    f_items_off = w;   w += csr * nitems;
    b_rowptr_off = w;  w += csr * (nrows + 1);
    b_entries_off = w; w += csr * (int64_t)nrows * n64;
    b_items_off = w;   w += csr * nitems;
    total_words = w;
    return true;
  }
  __host__ __device__ int32_t group_of(int32_t b, int32_t h) const {
    return (Bm == 1 ? 0 : b) * Hm + (Hm == 1 ? 0 : h);
  }
};

}  // namespace xsake
