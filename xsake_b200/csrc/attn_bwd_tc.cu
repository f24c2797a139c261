// HADS block-sparse attention backward on the sm_100a tensor cores (bf16 in and out, fp32
// accumulation in TMEM), head_dim 64, block sizes that are multiples of 64.
//
// The reference has no backward for its Pallas kernel; this is the gradient of
// sparse_attention_reference (kernels/pallas/sparse_attention.py:45-91).  With P the softmax of
// the masked, scaled scores and Dl_i = rowsum(dO_i * O_i):
//   dV = P^T dO,   dP = dO V^T,   dS = P * (dP - Dl),   dQ = scale * dS K,   dK = scale * dS^T Q
// A query row whose every key is masked attends uniformly to all S keys (the reference's
// finfo.min fill): it adds dO_row / S to every key's dV and nothing to dQ or dK (jnp.where
// passes no gradient to masked scores).
//
// Launches (all stream-ordered, deterministic: every output element is written by one thread
// from one fixed-order accumulation):
//   tc_bwd_prep_kernel  Dl and -lse*log2(e) per query row (8 lanes per row, 16-byte loads)
//   tc_ucol_kernel      (1/S) * sum of dO over fully masked rows, per (b, h) and column
//   tc_bwd_dkdv_kernel  work item = 128 keys (kv chunks 2u, 2u+1) of one (b, h), walking the
//                       64-query chunks that attend either half (the plan's transposed CSR).
//                       Per chunk: S^T = K Q^T and dP^T = V dO^T (tcgen05, M=128 N=64 K=64, fp32
//                       in TMEM); one thread per key row forms P^T and dS^T (bf16, shared
//                       memory, SWIZZLE_128B); dV += P^T dO and dK += dS^T Q accumulate in TMEM.
//   tc_bwd_dq_kernel    work item = 128 queries (q chunks 2t, 2t+1), walking their kv chunks
//                       (the forward CSR).  Per chunk: S = Q K^T and dP = dO V^T, one thread per
//                       query row forms dS, dQ += dS K.
// Roles in both (192 threads, two CTAs per SM, persistent over a longest-first item list taken
// from an atomic counter): warps 0-3 elementwise + epilogue (thread i = TMEM lane i = tile row
// i), warp 4 TMA producer, warp 5 MMA issuer (one elected lane).  TMEM (256 columns): the two
// score-like products at [0,64) and [64,128), the accumulators from 128.  The score buffers are
// single: the MMA of chunk i+1 is issued as soon as the elementwise warps have copied chunk i's
// rows into registers, so it overlaps their math.
#include "attn_common.cuh"
#include "sm100.cuh"

#include <algorithm>
#include <mutex>

XSAKE_DEFINE_DEVICE_ERROR(tcbwd)

namespace xsake {
namespace {

using namespace sm100;

constexpr int kThreads = 192;
constexpr int kTileBytes = 128 * 64 * 2;   // 128 rows x 64 bf16, SWIZZLE_128B
constexpr int kChunkBytes = 64 * 64 * 2;   // 64 rows
constexpr uint32_t kTmemCols = 256;
constexpr uint32_t kIdescQK = idesc_bf16(128, 64, false);   // A, B both K-major
constexpr uint32_t kIdescAcc = idesc_bf16(128, 64, true);   // B MN-major (rows of the K dimension)
constexpr int kItemReaders = 1 + 128;                       // MMA warp + elementwise threads

// ---- dK/dV kernel shared memory
// The per-query terms of P^T and dS^T enter through the tensor core: each chunk carries a bias
// operand of 64 query rows x 16 bf16 (SWIZZLE_32B) holding three bf16 parts of -lse/scale
// (elements 0-2) and of -Dl (elements 3-5), and two constant selector blocks of 128 key rows
// (ones at elements 0-2, resp. 3-5) turn one extra K=16 MMA per product into
// S^T + (-lse/scale) and dP^T - Dl, so the elementwise threads read no per-query values.
constexpr int kKvStages = 2;
constexpr int kBiasBytes = 64 * 32;                         // bias operand of one 64-query chunk
constexpr int kSelBytes = 128 * 32;                         // one selector block
constexpr int kKvStageBytes = 2 * kChunkBytes + kBiasBytes; // Q, dO, bias (1024-byte multiple)
constexpr int kOffK = 0, kOffV = kTileBytes, kOffPt = 2 * kTileBytes, kOffDSt = 3 * kTileBytes;
constexpr int kOffSel = 4 * kTileBytes;                     // selectors of the lse and Dl parts
constexpr int kOffKvRing = kOffSel + 2 * kSelBytes;
static_assert(kKvStageBytes % 1024 == 0 && kOffKvRing % 1024 == 0, "SWIZZLE_128B stage alignment");
constexpr int kOffKvBar = kOffKvRing + kKvStages * kKvStageBytes;

// ---- dQ kernel shared memory
constexpr int kQStages = 4;
constexpr int kQStageBytes = 2 * kChunkBytes;               // K, V
constexpr int kOffQ = 0, kOffDO = kTileBytes;
constexpr int kOffQRing = 2 * kTileBytes;
// dQ kernel TMEM: S [0, 64), dP [64, 128), dQ [128, 192), dS (bf16 pairs, the dQ MMA's A operand)
// double-buffered at [192, 224) and [224, 256).
constexpr uint32_t kDsCol = 192;
constexpr int kOffQBar = kOffQRing + kQStages * kQStageBytes;

template <int NS>
struct BwdBars {
  uint64_t item_full[2], item_empty[2];
  uint64_t tile_full, tile_empty;          // the resident 128-row operands of the item
  uint64_t ring_full[NS], ring_empty[NS];  // per-chunk operands
  uint64_t s_full, s_free;                 // score-like products in TMEM
  uint64_t p_full[2], p_free[2];           // bf16 operands written by the elementwise warps (dK/dV:
                                           // one buffer, index 0; dQ: dS buffers of even / odd steps)
  uint64_t acc_full, acc_free;             // accumulators of one item
  uint64_t drain;
};
constexpr int kKvSmemBytes = kOffKvBar + (int)sizeof(BwdBars<kKvStages>) + 64 + 1024;
constexpr int kQSmemBytes = kOffQBar + (int)sizeof(BwdBars<kQStages>) + 64 + 1024;
static_assert(2 * kKvSmemBytes <= 228 * 1024 - 2048, "two dK/dV CTAs per SM");
static_assert(2 * kQSmemBytes <= 228 * 1024 - 2048, "two dQ CTAs per SM");

struct BwdParams {
  AttnArgs a;
  float scale_log2;     // scale * log2(e)
  const float* nlse2;   // [B*H*S] -lse * log2(e); -inf for fully masked rows
  const uint8_t* bias;  // [B*H][S/64] bias operands of kBiasBytes (written by the prep kernel)
  int* counter;         // two work-item counters, zeroed by the host before the launches
};

__device__ __forceinline__ void fail(volatile int* abort, int detail) {
  if (atomicExch((int*)abort, 1) == 0) record_device_error(DEV_ERR_TIMEOUT, detail);
}

struct Item {
  int b, h, u, e0, n;
};

__device__ __forceinline__ Item decode(const AttnArgs& a, const int32_t* rowptr, int item) {
  const PlanLayout& L = a.L;
  Item it;
  it.u = item % L.npairs;
  const int bh = item / L.npairs;
  it.b = bh / a.H;
  it.h = bh % a.H;
  const int r = L.group_of(it.b, it.h) * L.npairs + it.u;
  it.e0 = rowptr[r];
  it.n = rowptr[r + 1] - it.e0;
  return it;
}

template <int NS>
__device__ void init_bars(BwdBars<NS>* bars) {
  for (int s = 0; s < 2; ++s) {
    mbar_init(&bars->item_full[s], 1);
    mbar_init(&bars->item_empty[s], kItemReaders);
  }
  mbar_init(&bars->tile_full, 1);
  mbar_init(&bars->tile_empty, 1);
  for (int s = 0; s < NS; ++s) {
    mbar_init(&bars->ring_full[s], 1);
    mbar_init(&bars->ring_empty[s], 1);
  }
  mbar_init(&bars->s_full, 1);
  mbar_init(&bars->s_free, 128);
  for (int b = 0; b < 2; ++b) {
    mbar_init(&bars->p_full[b], 128);
    mbar_init(&bars->p_free[b], 1);
  }
  mbar_init(&bars->acc_full, 1);
  mbar_init(&bars->acc_free, 128);
  mbar_init(&bars->drain, 1);
  fence_barrier_init();
  fence_proxy_async_smem();
}

// Work-item distribution shared by both kernels: the producer warp takes item indices from the
// global counter and publishes the item through a 2-slot ring read by the MMA warp and the
// elementwise threads.  Returns the item (-1 = no more work) or -2 on a failed wait.
template <int NS>
__device__ __forceinline__ int publish_item(BwdBars<NS>* bars, volatile int* item_slot, uint32_t k,
                                            int* counter, const int32_t* items, int nitems, volatile int* abort) {
  const int lane = threadIdx.x & 31;
  const int slot = k & 1;
  if (!warp_mbar_wait(&bars->item_empty[slot], ((k >> 1) & 1) ^ 1, abort)) return -2;
  int idx = 0;
  if (lane == 0) idx = *abort ? nitems : atomicAdd(counter, 1);
  idx = __shfl_sync(0xffffffffu, idx, 0);
  const int item = idx < nitems ? items[idx] : -1;
  if (elect_one()) {
    item_slot[slot] = item;
    mbar_arrive(&bars->item_full[slot]);
  }
  __syncwarp();
  return item;
}

template <int NS>
__device__ __forceinline__ int take_item(BwdBars<NS>* bars, volatile int* item_slot, uint32_t k, bool one_lane,
                                         volatile int* abort) {
  const int slot = k & 1;
  if (!warp_mbar_wait(&bars->item_full[slot], (k >> 1) & 1, abort)) return -2;
  const int item = item_slot[slot];
  __syncwarp();
  if (one_lane) {
    if (elect_one()) mbar_arrive(&bars->item_empty[slot]);
    __syncwarp();
  } else {
    mbar_arrive(&bars->item_empty[slot]);
  }
  return item;
}

// Bounded wait for copies still in flight before a failing CTA exits.
template <int NS>
__device__ void drain_copies(BwdBars<NS>* bars) {
  for (int s = 0; s < NS; ++s) {
    const uint64_t t0 = global_timer_ns();
    while (!mbar_try_wait(&bars->ring_full[s], 0) && !mbar_try_wait(&bars->ring_full[s], 1) &&
           global_timer_ns() - t0 < 1000000ull) {
    }
  }
}

template <int NS>
__device__ void drain_mma(BwdBars<NS>* bars) {
  const int lane = threadIdx.x & 31;
  if (elect_one()) mma_commit(&bars->drain);
  __syncwarp();
  if (lane == 0) {
    const uint64_t t0 = global_timer_ns();
    while (!mbar_try_wait(&bars->drain, 0) && global_timer_ns() - t0 < kWaitLimitNs) {
    }
  }
  __syncwarp();
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 b = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&b);
}

// Writes one 64-wide bf16 row of a SWIZZLE_128B operand tile: 16-byte chunk cc of row r lives
// at (r / 8) * 1024 + (r % 8) * 128 + ((cc ^ (r % 8)) * 16).
__device__ __forceinline__ void store_sw128_half(uint8_t* rowp, int rsw, int hh, const uint32_t* pk16) {
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const int cc = 4 * hh + c;
    *reinterpret_cast<uint4*>(rowp + ((cc ^ rsw) << 4)) =
        make_uint4(pk16[4 * c], pk16[4 * c + 1], pk16[4 * c + 2], pk16[4 * c + 3]);
  }
}

// =============================================================================== dK / dV
__global__ void __launch_bounds__(kThreads, 2)
tc_bwd_dkdv_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                   const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmDO,
                   const BwdParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  using Bars = BwdBars<kKvStages>;
  Bars* bars = reinterpret_cast<Bars*>(smem + kOffKvBar);
  uint8_t* misc = smem + kOffKvBar + sizeof(Bars);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(misc);
  volatile int* abort = reinterpret_cast<volatile int*>(misc + 4);
  volatile int* plan_ok = reinterpret_cast<volatile int*>(misc + 8);
  volatile int* item_slot = reinterpret_cast<volatile int*>(misc + 16);   // [2]
  const AttnArgs& a = p.a;
  const PlanLayout& L = a.L;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    *abort = 0;
    *plan_ok = plan_matches(a) && a.plan[H_HAS_CSR] == 1;
    if (!*plan_ok) record_device_error(DEV_ERR_PLAN, 20);
    init_bars(bars);
  }
  if (threadIdx.x < 128) {
    // Selector rows, the same for every key row: bf16 1.0 at elements 0-2 (first block) and 3-5.
    constexpr uint32_t kOne = 0x3F80u;
    const int r = threadIdx.x;
    uint8_t* sel = smem + kOffSel;
    *reinterpret_cast<uint4*>(sel + sw32_offset(r, 0)) = make_uint4(kOne | (kOne << 16), kOne, 0u, 0u);
    *reinterpret_cast<uint4*>(sel + sw32_offset(r, 1)) = make_uint4(0u, 0u, 0u, 0u);
    *reinterpret_cast<uint4*>(sel + kSelBytes + sw32_offset(r, 0)) =
        make_uint4(0u, kOne << 16, kOne | (kOne << 16), 0u);
    *reinterpret_cast<uint4*>(sel + kSelBytes + sw32_offset(r, 1)) = make_uint4(0u, 0u, 0u, 0u);
    fence_proxy_async_smem();   // generic-proxy writes read by the tensor core
  }
  if (warp == 4 && lane == 0) {
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmDO);
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int32_t* rowptr = a.plan + L.b_rowptr_off;
  const int32_t* entries = a.plan + L.b_entries_off;
  const int32_t* items = a.plan + L.b_items_off;

  if (*plan_ok) {
    if (warp == 4) {
      // ------------------------------------------------------------------ TMA producer
      uint32_t g = 0, j = 0;
      bool ok = true;
      for (uint32_t k = 0; ok; ++k) {
        const int item = publish_item(bars, item_slot, k, p.counter, items, a.plan[H_B_ITEMS], abort);
        if (item == -2) { ok = false; break; }
        if (item < 0) break;
        const Item w = decode(a, rowptr, item);
        if (w.n == 0) continue;
        if (j > 0 && !warp_mbar_wait(&bars->tile_empty, (j - 1) & 1, abort)) { ok = false; break; }
        if (elect_one()) {
          mbar_arrive_expect_tx(&bars->tile_full, 2 * kTileBytes);
          tma_load_4d(smem + kOffK, &tmK, &bars->tile_full, 0, 128 * w.u, w.h, w.b);
          tma_load_4d(smem + kOffV, &tmV, &bars->tile_full, 0, 128 * w.u, w.h, w.b);
        }
        __syncwarp();
        ++j;
        const uint8_t* bias = p.bias + (int64_t)(w.b * a.H + w.h) * (a.S / 64) * kBiasBytes;
        for (int i = 0; i < w.n; ++i, ++g) {
          const int c = entries[w.e0 + i] & kEntryIdxMask;
          const int st = g % kKvStages;
          if (!warp_mbar_wait(&bars->ring_empty[st], ((g / kKvStages) & 1) ^ 1, abort)) { ok = false; break; }
          if (elect_one()) {
            uint8_t* sb = smem + kOffKvRing + st * kKvStageBytes;
            mbar_arrive_expect_tx(&bars->ring_full[st], 2 * kChunkBytes + kBiasBytes);
            tma_load_4d(sb, &tmQ, &bars->ring_full[st], 0, 64 * c, w.h, w.b);
            tma_load_4d(sb + kChunkBytes, &tmDO, &bars->ring_full[st], 0, 64 * c, w.h, w.b);
            bulk_load(sb + 2 * kChunkBytes, bias + (int64_t)c * kBiasBytes, kBiasBytes, &bars->ring_full[st]);
          }
          __syncwarp();
        }
      }
      if (!ok && lane == 0) {
        fail(abort, 21);
        drain_copies(bars);
      }
      __syncwarp();
    } else if (warp == 5) {
      // ------------------------------------------------------------------ MMA issuer
      // Chunk i+1's S^T / dP^T are issued once the elementwise warps have read chunk i's, and
      // before chunk i's accumulation (which waits for its P^T / dS^T in shared memory).
      const uint64_t kdesc = sw128_desc(smem_u32(smem + kOffK), 16, 1024);
      const uint64_t vdesc = sw128_desc(smem_u32(smem + kOffV), 16, 1024);
      const uint64_t ptdesc = sw128_desc(smem_u32(smem + kOffPt), 16, 1024);
      const uint64_t dstdesc = sw128_desc(smem_u32(smem + kOffDSt), 16, 1024);
      const uint64_t ring0 = sw128_desc(smem_u32(smem + kOffKvRing), 16, 1024);
      const uint64_t sel_lse = sw32_desc(smem_u32(smem + kOffSel), 256);
      const uint64_t sel_dl = sw32_desc(smem_u32(smem + kOffSel + kSelBytes), 256);
      const uint64_t bias0 = sw32_desc(smem_u32(smem + kOffKvRing + 2 * kChunkBytes), 256);
      uint32_t g = 0, j = 0;
      bool ok = true;
      auto issue_scores = [&](uint32_t gs) -> bool {
        const int st = gs % kKvStages;
        if (gs > 0 && !warp_mbar_wait(&bars->s_free, (gs - 1) & 1, abort)) return false;
        if (!warp_mbar_wait(&bars->ring_full[st], (gs / kKvStages) & 1, abort)) return false;
        tc_fence_after();
        if (elect_one()) {
          const uint64_t qd = ring0 + (uint64_t)((st * kKvStageBytes) >> 4);
          const uint64_t dod = ring0 + (uint64_t)((st * kKvStageBytes + kChunkBytes) >> 4);
          const uint64_t bd = bias0 + (uint64_t)((st * kKvStageBytes) >> 4);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) mma_bf16_ss(tmem + 0, kdesc + 2 * kk, qd + 2 * kk, kIdescQK, kk > 0);
          mma_bf16_ss(tmem + 0, sel_lse, bd, kIdescQK, 1u);   // + (-lse / scale)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) mma_bf16_ss(tmem + 64, vdesc + 2 * kk, dod + 2 * kk, kIdescQK, kk > 0);
          mma_bf16_ss(tmem + 64, sel_dl, bd, kIdescQK, 1u);   // - Dl
          mma_commit(&bars->s_full);
        }
        __syncwarp();
        return true;
      };
      auto issue_acc = [&](uint32_t gs, bool first) -> bool {
        const int st = gs % kKvStages;
        if (!warp_mbar_wait(&bars->p_full[0], gs & 1, abort)) return false;
        if (first && j > 0 && !warp_mbar_wait(&bars->acc_free, (j - 1) & 1, abort)) return false;
        tc_fence_after();
        if (elect_one()) {
          const uint64_t qd = ring0 + (uint64_t)((st * kKvStageBytes) >> 4);
          const uint64_t dod = ring0 + (uint64_t)((st * kKvStageBytes + kChunkBytes) >> 4);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)   // dV += P^T dO
            mma_bf16_ss(tmem + 128, ptdesc + 2 * kk, dod + (uint64_t)((2048 * kk) >> 4), kIdescAcc,
                        (first && kk == 0) ? 0u : 1u);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)   // dK += dS^T Q
            mma_bf16_ss(tmem + 192, dstdesc + 2 * kk, qd + (uint64_t)((2048 * kk) >> 4), kIdescAcc,
                        (first && kk == 0) ? 0u : 1u);
          mma_commit(&bars->p_free[0]);
          mma_commit(&bars->ring_empty[st]);
        }
        __syncwarp();
        return true;
      };
      for (uint32_t k = 0; ok; ++k) {
        const int item = take_item(bars, item_slot, k, true, abort);
        if (item == -2) { ok = false; break; }
        if (item < 0) break;
        const Item w = decode(a, rowptr, item);
        if (w.n == 0) continue;
        if (!warp_mbar_wait(&bars->tile_full, j & 1, abort)) { ok = false; break; }
        if (!issue_scores(g)) { ok = false; break; }
        for (int i = 0; i < w.n && ok; ++i) {
          if (i + 1 < w.n && !issue_scores(g + i + 1)) { ok = false; break; }
          if (!issue_acc(g + i, i == 0)) { ok = false; break; }
        }
        if (!ok) break;
        g += w.n;
        if (elect_one()) {
          mma_commit(&bars->acc_full);
          mma_commit(&bars->tile_empty);
        }
        __syncwarp();
        ++j;
      }
      if (!ok && lane == 0) fail(abort, 22);
      drain_mma(bars);
    } else {
      // ------------------------------------------------------------------ elementwise + epilogue
      const int row = threadIdx.x;             // key row of the tile = TMEM lane
      const int half = row >> 6, kl = row & 63;
      const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
      const int32_t f_active = half ? kFlagActive1 : kFlagActive0;
      const int32_t f_diag = half ? kFlagDiag1 : kFlagDiag0;
      const int rsw = row & 7;
      uint8_t* ptrow = smem + kOffPt + (row >> 3) * 1024 + rsw * 128;
      uint8_t* dsrow = smem + kOffDSt + (row >> 3) * 1024 + rsw * 128;
      const uint64_t cc2 = pk2(p.scale_log2, p.scale_log2);
      uint32_t g = 0, j = 0;
      bool ok = true;
      for (uint32_t k = 0; ok; ++k) {
        const int item = take_item(bars, item_slot, k, false, abort);
        if (item == -2) { ok = false; break; }
        if (item < 0) break;
        const Item w = decode(a, rowptr, item);
        if (w.n > 0) {
          for (int i = 0; i < w.n; ++i, ++g) {
            const int32_t e = entries[w.e0 + i];
            // S^T - lse/scale and dP^T - Dl (the bias MMAs): nothing per query is read here.
            if (!warp_mbar_wait(&bars->s_full, g & 1, abort)) { ok = false; break; }
            tc_fence_after();
            const bool act = (e & f_active) != 0;    // warp-uniform (a warp is inside one half)
            const bool dg = (e & f_diag) != 0;
            uint32_t ppa[2][16], pda[2][16];   // P^T and dS^T of this row, bf16 pairs
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
              uint32_t* pp = ppa[hh];
              uint32_t* pd = pda[hh];
              uint32_t sr[32], dr[32];   // half hh of S^T and dP^T: 64 registers live instead of 128
              XSAKE_TMEM_LD32(tmem + lane_base + 32 * hh, sr);
              XSAKE_TMEM_LD32(tmem + lane_base + 64 + 32 * hh, dr);
              XSAKE_TMEM_WAIT_LD32(sr);
              XSAKE_TMEM_WAIT_LD32(dr);
              if (hh == 1) {
                tc_fence_before();
                mbar_arrive(&bars->s_free);
              }
              if (act) {
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                  const int jq = 32 * hh + 4 * q;   // query index within the chunk
                  const int j0 = 4 * q;             // index within this half's registers
                  float x0, x1, x2, x3;
                  upk2(mul2(pk2(__uint_as_float(sr[j0]), __uint_as_float(sr[j0 + 1])), cc2), x0, x1);
                  upk2(mul2(pk2(__uint_as_float(sr[j0 + 2]), __uint_as_float(sr[j0 + 3])), cc2), x2, x3);
                  float p0 = ex2(x0), p1 = ex2(x1), p2 = ex2(x2), p3 = ex2(x3);
                  if (dg) {   // token-level causal cut: key kl is after query j
                    if (jq < kl) p0 = 0.f;
                    if (jq + 1 < kl) p1 = 0.f;
                    if (jq + 2 < kl) p2 = 0.f;
                    if (jq + 3 < kl) p3 = 0.f;
                  }
                  float d0, d1, d2, d3;
                  upk2(mul2(pk2(p0, p1), pk2(__uint_as_float(dr[j0]), __uint_as_float(dr[j0 + 1]))), d0, d1);
                  upk2(mul2(pk2(p2, p3), pk2(__uint_as_float(dr[j0 + 2]), __uint_as_float(dr[j0 + 3]))), d2, d3);
                  pp[2 * q] = pack_bf16(p0, p1);
                  pp[2 * q + 1] = pack_bf16(p2, p3);
                  pd[2 * q] = pack_bf16(d0, d1);
                  pd[2 * q + 1] = pack_bf16(d2, d3);
                }
              } else {
#pragma unroll
                for (int q = 0; q < 16; ++q) pp[q] = pd[q] = 0u;
              }
            }
            // Computed into registers first: the wait for the previous chunk's accumulation to
            // release P^T / dS^T overlaps the exponentials above.
            if (g > 0 && !warp_mbar_wait(&bars->p_free[0], (g - 1) & 1, abort)) { ok = false; break; }
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
              store_sw128_half(ptrow, rsw, hh, ppa[hh]);
              store_sw128_half(dsrow, rsw, hh, pda[hh]);
            }
            fence_proxy_async_smem();
            tc_fence_before();
            mbar_arrive(&bars->p_full[0]);
          }
          if (!ok) break;
          if (!warp_mbar_wait(&bars->acc_full, j & 1, abort)) { ok = false; break; }
          tc_fence_after();
        }
        // ---------------------------------------------------------------- epilogue
        // 32 columns of dV and dK at a time; the accumulators are released after the last load.
        const int key = 128 * w.u + row;
        const int64_t bh = (int64_t)w.b * a.H + w.h;
        const float4* uc = reinterpret_cast<const float4*>(a.ucol + bh * 64);
        const int64_t goff = w.b * a.os[0] + w.h * a.os[1] + (int64_t)(key < a.S ? key : 0) * a.os[2];
        uint4* dvg = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(a.dv) + goff);
        uint4* dkg = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(a.dk) + goff);
#pragma unroll
        for (int hc = 0; hc < 2; ++hc) {
          uint32_t accv[32], acck[32];
          if (w.n > 0) {
            XSAKE_TMEM_LD32(tmem + lane_base + 128 + 32 * hc, accv);
            XSAKE_TMEM_LD32(tmem + lane_base + 192 + 32 * hc, acck);
            XSAKE_TMEM_WAIT_LD32(accv);
            XSAKE_TMEM_WAIT_LD32(acck);
          } else {
#pragma unroll
            for (int c = 0; c < 32; ++c) accv[c] = acck[c] = 0u;
          }
          if (key < a.S) {
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              const float4 u0 = uc[8 * hc + 2 * c], u1 = uc[8 * hc + 2 * c + 1];
              const float* v = reinterpret_cast<const float*>(accv + 8 * c);
              const float* kk = reinterpret_cast<const float*>(acck + 8 * c);
              dvg[4 * hc + c] = make_uint4(pack_bf16(v[0] + u0.x, v[1] + u0.y), pack_bf16(v[2] + u0.z, v[3] + u0.w),
                                           pack_bf16(v[4] + u1.x, v[5] + u1.y), pack_bf16(v[6] + u1.z, v[7] + u1.w));
              dkg[4 * hc + c] =
                  make_uint4(pack_bf16(kk[0] * a.scale, kk[1] * a.scale), pack_bf16(kk[2] * a.scale, kk[3] * a.scale),
                             pack_bf16(kk[4] * a.scale, kk[5] * a.scale), pack_bf16(kk[6] * a.scale, kk[7] * a.scale));
            }
          }
        }
        if (w.n > 0) {
          tc_fence_before();
          mbar_arrive(&bars->acc_free);
          ++j;
        }
      }
      if (!ok) fail(abort, 23);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// =============================================================================== dQ
__global__ void __launch_bounds__(kThreads, 2)
tc_bwd_dq_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmDO,
                 const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                 const BwdParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  using Bars = BwdBars<kQStages>;
  Bars* bars = reinterpret_cast<Bars*>(smem + kOffQBar);
  uint8_t* misc = smem + kOffQBar + sizeof(Bars);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(misc);
  volatile int* abort = reinterpret_cast<volatile int*>(misc + 4);
  volatile int* plan_ok = reinterpret_cast<volatile int*>(misc + 8);
  volatile int* item_slot = reinterpret_cast<volatile int*>(misc + 16);   // [2]
  const AttnArgs& a = p.a;
  const PlanLayout& L = a.L;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    *abort = 0;
    *plan_ok = plan_matches(a) && a.plan[H_HAS_CSR] == 1;
    if (!*plan_ok) record_device_error(DEV_ERR_PLAN, 30);
    init_bars(bars);
  }
  if (warp == 4 && lane == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmDO);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int32_t* rowptr = a.plan + L.f_rowptr_off;
  const int32_t* entries = a.plan + L.f_entries_off;
  const int32_t* items = a.plan + L.f_items_off;

  if (*plan_ok) {
    if (warp == 4) {
      // ------------------------------------------------------------------ TMA producer
      uint32_t g = 0, j = 0;
      bool ok = true;
      for (uint32_t k = 0; ok; ++k) {
        const int item = publish_item(bars, item_slot, k, p.counter + 1, items, a.plan[H_F_ITEMS], abort);
        if (item == -2) { ok = false; break; }
        if (item < 0) break;
        const Item w = decode(a, rowptr, item);
        if (w.n == 0) continue;
        if (j > 0 && !warp_mbar_wait(&bars->tile_empty, (j - 1) & 1, abort)) { ok = false; break; }
        if (elect_one()) {
          mbar_arrive_expect_tx(&bars->tile_full, 2 * kTileBytes);
          tma_load_4d(smem + kOffQ, &tmQ, &bars->tile_full, 0, 128 * w.u, w.h, w.b);
          tma_load_4d(smem + kOffDO, &tmDO, &bars->tile_full, 0, 128 * w.u, w.h, w.b);
        }
        __syncwarp();
        ++j;
        for (int i = 0; i < w.n; ++i, ++g) {
          const int c = entries[w.e0 + i] & kEntryIdxMask;
          const int st = g % kQStages;
          if (!warp_mbar_wait(&bars->ring_empty[st], ((g / kQStages) & 1) ^ 1, abort)) { ok = false; break; }
          if (elect_one()) {
            uint8_t* sb = smem + kOffQRing + st * kQStageBytes;
            mbar_arrive_expect_tx(&bars->ring_full[st], 2 * kChunkBytes);
            tma_load_4d(sb, &tmK, &bars->ring_full[st], 0, 64 * c, w.h, w.b);
            tma_load_4d(sb + kChunkBytes, &tmV, &bars->ring_full[st], 0, 64 * c, w.h, w.b);
          }
          __syncwarp();
        }
      }
      if (!ok && lane == 0) {
        fail(abort, 31);
        drain_copies(bars);
      }
      __syncwarp();
    } else if (warp == 5) {
      // ------------------------------------------------------------------ MMA issuer
      const uint64_t qdesc = sw128_desc(smem_u32(smem + kOffQ), 16, 1024);
      const uint64_t dodesc = sw128_desc(smem_u32(smem + kOffDO), 16, 1024);
      const uint64_t ring0 = sw128_desc(smem_u32(smem + kOffQRing), 16, 1024);
      uint32_t g = 0, j = 0;
      bool ok = true;
      auto issue_scores = [&](uint32_t gs) -> bool {
        const int st = gs % kQStages;
        if (gs > 0 && !warp_mbar_wait(&bars->s_free, (gs - 1) & 1, abort)) return false;
        if (!warp_mbar_wait(&bars->ring_full[st], (gs / kQStages) & 1, abort)) return false;
        tc_fence_after();
        if (elect_one()) {
          const uint64_t kd = ring0 + (uint64_t)((st * kQStageBytes) >> 4);
          const uint64_t vd = ring0 + (uint64_t)((st * kQStageBytes + kChunkBytes) >> 4);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) mma_bf16_ss(tmem + 0, qdesc + 2 * kk, kd + 2 * kk, kIdescQK, kk > 0);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) mma_bf16_ss(tmem + 64, dodesc + 2 * kk, vd + 2 * kk, kIdescQK, kk > 0);
          mma_commit(&bars->s_full);
        }
        __syncwarp();
        return true;
      };
      auto issue_acc = [&](uint32_t gs, bool first) -> bool {
        const int st = gs % kQStages;
        // dS of step gs sits in TMEM buffer gs & 1; each buffer's barriers complete once per two
        // steps, so their parity waits stay unambiguous with the elementwise warps a step ahead.
        if (!warp_mbar_wait(&bars->p_full[gs & 1], (gs >> 1) & 1, abort)) return false;
        if (first && j > 0 && !warp_mbar_wait(&bars->acc_free, (j - 1) & 1, abort)) return false;
        tc_fence_after();
        if (elect_one()) {
          const uint64_t kd = ring0 + (uint64_t)((st * kQStageBytes) >> 4);
          const uint32_t ds = tmem + kDsCol + 32 * (gs & 1);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)   // dQ += dS K, dS (A) from TMEM
            mma_bf16_ts(tmem + 128, ds + 8 * kk, kd + (uint64_t)((2048 * kk) >> 4), kIdescAcc,
                        (first && kk == 0) ? 0u : 1u);
          mma_commit(&bars->p_free[gs & 1]);
          mma_commit(&bars->ring_empty[st]);
        }
        __syncwarp();
        return true;
      };
      for (uint32_t k = 0; ok; ++k) {
        const int item = take_item(bars, item_slot, k, true, abort);
        if (item == -2) { ok = false; break; }
        if (item < 0) break;
        const Item w = decode(a, rowptr, item);
        if (w.n == 0) continue;
        if (!warp_mbar_wait(&bars->tile_full, j & 1, abort)) { ok = false; break; }
        if (!issue_scores(g)) { ok = false; break; }
        for (int i = 0; i < w.n && ok; ++i) {
          if (i + 1 < w.n && !issue_scores(g + i + 1)) { ok = false; break; }
          if (!issue_acc(g + i, i == 0)) { ok = false; break; }
        }
        if (!ok) break;
        g += w.n;
        if (elect_one()) {
          mma_commit(&bars->acc_full);
          mma_commit(&bars->tile_empty);
        }
        __syncwarp();
        ++j;
      }
      if (!ok && lane == 0) fail(abort, 32);
      drain_mma(bars);
    } else {
      // ------------------------------------------------------------------ elementwise + epilogue
      const int row = threadIdx.x;             // query row of the tile = TMEM lane
      const int half = row >> 6, ql = row & 63;
      const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
      const int32_t f_active = half ? kFlagActive1 : kFlagActive0;
      const int32_t f_diag = half ? kFlagDiag1 : kFlagDiag0;
      const uint64_t cc2 = pk2(p.scale_log2, p.scale_log2);
      uint32_t g = 0, j = 0;
      bool ok = true;
      for (uint32_t k = 0; ok; ++k) {
        const int item = take_item(bars, item_slot, k, false, abort);
        if (item == -2) { ok = false; break; }
        if (item < 0) break;
        const Item w = decode(a, rowptr, item);
        const int tok = 128 * w.u + row;
        const bool valid = tok < a.S;
        const int64_t rix = ((int64_t)w.b * a.H + w.h) * a.S + (valid ? tok : 0);
        uint32_t accq[64];
        if (w.n > 0) {
          const float nl = valid ? p.nlse2[rix] : -INFINITY;
          const float dl = valid ? a.delta[rix] : 0.f;
          const uint64_t nl2 = pk2(nl, nl), dl2 = pk2(dl, dl);
          for (int i = 0; i < w.n; ++i, ++g) {
            const int32_t e = entries[w.e0 + i];
            if (!warp_mbar_wait(&bars->s_full, g & 1, abort)) { ok = false; break; }
            tc_fence_after();
            const bool act = (e & f_active) != 0;    // warp-uniform
            const bool dg = (e & f_diag) != 0;
            uint32_t pda[2][16];   // dS of this row, bf16 pairs
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
              uint32_t* pd = pda[hh];
              uint32_t sr[32], dr[32];   // half hh of S and dP: 64 registers live instead of 128
              XSAKE_TMEM_LD32(tmem + lane_base + 32 * hh, sr);
              XSAKE_TMEM_LD32(tmem + lane_base + 64 + 32 * hh, dr);
              XSAKE_TMEM_WAIT_LD32(sr);
              XSAKE_TMEM_WAIT_LD32(dr);
              if (hh == 1) {
                tc_fence_before();
                mbar_arrive(&bars->s_free);
              }
              if (act) {
#pragma unroll
                for (int q = 0; q < 16; ++q) {
                  const int jk = 32 * hh + 2 * q;   // key index within the chunk
                  const int j0 = 2 * q;             // index within this half's registers
                  float x0, x1;
                  upk2(fma2(pk2(__uint_as_float(sr[j0]), __uint_as_float(sr[j0 + 1])), cc2, nl2), x0, x1);
                  float p0 = ex2(x0), p1 = ex2(x1);
                  if (dg) {   // token-level causal cut: key j is after query ql
                    if (jk > ql) p0 = 0.f;
                    if (jk + 1 > ql) p1 = 0.f;
                  }
                  float d0, d1;
                  upk2(mul2(pk2(p0, p1), sub2(pk2(__uint_as_float(dr[j0]), __uint_as_float(dr[j0 + 1])), dl2)), d0, d1);
                  pd[q] = pack_bf16(d0, d1);
                }
              } else {
#pragma unroll
                for (int q = 0; q < 16; ++q) pd[q] = 0u;
              }
            }
            // Computed into registers first; the dS buffer of this step was last read by the dQ
            // MMA of step g - 2.
            if (g > 1 && !warp_mbar_wait(&bars->p_free[g & 1], ((g - 2) >> 1) & 1, abort)) { ok = false; break; }
            const uint32_t ds = tmem + lane_base + kDsCol + 32 * (g & 1);
            XSAKE_TMEM_ST16(ds, pda[0]);
            XSAKE_TMEM_ST16(ds + 16, pda[1]);
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(&bars->p_full[g & 1]);
          }
          if (!ok) break;
          if (!warp_mbar_wait(&bars->acc_full, j & 1, abort)) { ok = false; break; }
          tc_fence_after();
          XSAKE_TMEM_LD32(tmem + lane_base + 128, accq);
          XSAKE_TMEM_LD32(tmem + lane_base + 160, (accq + 32));
          XSAKE_TMEM_WAIT_LD32(accq);
          XSAKE_TMEM_WAIT_LD32((accq + 32));
          tc_fence_before();
          mbar_arrive(&bars->acc_free);
          ++j;
        } else {
#pragma unroll
          for (int c = 0; c < 64; ++c) accq[c] = 0u;
        }
        if (valid) {
          uint4* dqg = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(a.dq) + w.b * a.os[0] +
                                                w.h * a.os[1] + (int64_t)tok * a.os[2]);
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            const float* v = reinterpret_cast<const float*>(accq + 8 * c);
            dqg[c] = make_uint4(pack_bf16(v[0] * a.scale, v[1] * a.scale), pack_bf16(v[2] * a.scale, v[3] * a.scale),
                                pack_bf16(v[4] * a.scale, v[5] * a.scale), pack_bf16(v[6] * a.scale, v[7] * a.scale));
          }
        }
      }
      if (!ok) fail(abort, 33);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// =============================================================================== prep
// Three bf16 parts whose sum is v to within fp32 rounding (each part takes the remainder).
__device__ __forceinline__ void split3_bf16(float v, uint32_t (&h)[3]) {
#pragma unroll
  for (int i = 0; i < 3; ++i) {
    const __nv_bfloat16 b = __float2bfloat16_rn(v);
    h[i] = (uint32_t)__bfloat16_as_ushort(b);
    v -= __bfloat162float(b);
  }
}

// Dl = rowsum(dO * O) and -lse * log2(e) (-inf for fully masked rows, whose lse is the
// finfo.min fill) for every query row, and the row's line of its chunk's bias operand (the dK/dV
// kernel's extra MMAs): parts of -lse/scale at elements 0-2 (-1e30 for fully masked rows, finite
// so that the selector's zeros never multiply an infinity) and of -Dl at 3-5; 8 lanes per row,
// one 16-byte load of O and dO each.
__global__ void __launch_bounds__(256) tc_bwd_prep_kernel(AttnArgs a, float* __restrict__ nlse2,
                                                          uint8_t* __restrict__ bias) {
  const int64_t nrows = (int64_t)a.B * a.H * a.S;
  const int64_t row = (int64_t)blockIdx.x * 32 + (threadIdx.x >> 3);
  const int sub = threadIdx.x & 7;
  float acc = 0.f;
  if (row < nrows) {
    const int s = (int)(row % a.S);
    const int64_t bh = row / a.S;
    const int b = (int)(bh / a.H), h = (int)(bh % a.H);
    if (!plan_unit_selected(a.plan, a.L, b, h)) return;   // warp-uniform: 4 rows of one unit
    const int64_t off = b * a.os[0] + h * a.os[1] + (int64_t)s * a.os[2] + 8 * sub;
    const uint4 o = *reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(a.o) + off);
    const uint4 d = *reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(a.dout) + off);
    const uint32_t ow[4] = {o.x, o.y, o.z, o.w}, dw[4] = {d.x, d.y, d.z, d.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 of = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&ow[i]));
      const float2 df = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&dw[i]));
      acc = fmaf(of.x, df.x, acc);
      acc = fmaf(of.y, df.y, acc);
    }
  }
  acc += __shfl_xor_sync(0xffffffffu, acc, 1);
  acc += __shfl_xor_sync(0xffffffffu, acc, 2);
  acc += __shfl_xor_sync(0xffffffffu, acc, 4);
  if (row < nrows && sub == 0) {
    a.delta[row] = acc;
    const float l = a.lse[row];
    const bool empty = l == kMaskFill;
    nlse2[row] = empty ? -INFINITY : -l * kLog2e;
    uint32_t hl[3], hd[3];
    split3_bf16(empty ? -1e30f : -l / a.scale, hl);
    split3_bf16(-acc, hd);
    uint8_t* line = bias + (row >> 6) * kBiasBytes;   // S is a multiple of 64 on this path
    const int r = (int)(row & 63);
    *reinterpret_cast<uint4*>(line + sw32_offset(r, 0)) =
        make_uint4(hl[0] | (hl[1] << 16), hl[2] | (hd[0] << 16), hd[1] | (hd[2] << 16), 0u);
    *reinterpret_cast<uint4*>(line + sw32_offset(r, 1)) = make_uint4(0u, 0u, 0u, 0u);
  }
}

// ucol[b, h, d] = (1/S) * sum of dO over the rows of fully masked q-blocks (0 when none).
__global__ void __launch_bounds__(64) tc_ucol_kernel(AttnArgs a) {
  const int bh = blockIdx.x, b = bh / a.H, h = bh % a.H;
  if (!plan_unit_selected(a.plan, a.L, b, h)) return;
  const int c = threadIdx.x;
  const uint8_t* qe =
      reinterpret_cast<const uint8_t*>(a.plan + a.L.qempty_off) + (int64_t)a.L.group_of(b, h) * a.L.nq;
  float acc = 0.f;
  for (int qb = 0; qb < a.L.nq; ++qb) {
    if (!qe[qb]) continue;
    for (int r = qb * a.L.bs; r < (qb + 1) * a.L.bs; ++r)
      acc += __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(a.dout)[b * a.os[0] + h * a.os[1] +
                                                                             (int64_t)r * a.os[2] + c]);
  }
  a.ucol[(int64_t)bh * 64 + c] = acc / (float)a.S;
}

constexpr int kMaxDev = 64;
std::once_flag g_attr_once[kMaxDev];
cudaError_t g_attr_err[kMaxDev];

}  // namespace

bool tc_attn_bwd_supported(const AttnArgs& a, int dtype) {
  if (!tc_attn_fwd_supported(a, dtype)) return false;
  auto al = [](const void* ptr) { return ((uintptr_t)ptr & 15) == 0; };
  if (!(al(a.dout) && al(a.dq) && al(a.dk) && al(a.dv))) return false;
  CUtensorMap m;
  const bool ok = tc_make_map(&m, a.dout, a.os, a.B, a.H, a.S, 128) == XSAKE_OK;
  clear_error();
  return ok;
}

// Workspace: delta [B*H*S] | ucol [B*H*64] | -lse*log2e [B*H*S] | counters (256 B) | bias
// operands [B*H*S/64][kBiasBytes]; each section 256-byte aligned (the first two are shared with
// the CUDA-core backward).
int tc_attn_bwd(const AttnArgs& a_in, void* ws, size_t ws_bytes, cudaStream_t s) {
  DeviceInfo di;
  int st = device_info(&di);
  if (st) return st;
  XSAKE_REQUIRE(di.major == 10, XSAKE_EUNSUPPORTED, "tensor-core path needs sm_100 (got sm_%d%d)", di.major,
                di.minor);
  AttnArgs a = a_in;
  const int64_t bh = (int64_t)a.B * a.H;
  const size_t s1 = align_up((size_t)(bh * a.S) * 4, 256), s2 = align_up((size_t)(bh * a.D) * 4, 256);
  const size_t s_bias = (size_t)(bh * (a.S / 64)) * kBiasBytes;
  const size_t need = 2 * s1 + s2 + 256 + s_bias;
  XSAKE_REQUIRE(ws != nullptr && ((uintptr_t)ws & 255) == 0 && ws_bytes >= need, XSAKE_EINVAL,
                "the tensor-core backward needs a 256-byte aligned workspace of %zu bytes (got %zu)", need,
                ws_bytes);
  uint8_t* w = reinterpret_cast<uint8_t*>(ws);
  a.delta = reinterpret_cast<float*>(w);
  a.ucol = reinterpret_cast<float*>(w + s1);
  float* nlse2 = reinterpret_cast<float*>(w + s1 + s2);
  int* counters = reinterpret_cast<int*>(w + 2 * s1 + s2);
  uint8_t* bias = w + 2 * s1 + s2 + 256;

  CUtensorMap mq, mk, mv, mdo, mq128, mdo128, mk128, mv128;
  if ((st = tc_make_map(&mq, a.q, a.qs, a.B, a.H, a.S, 64))) return st;
  if ((st = tc_make_map(&mdo, a.dout, a.os, a.B, a.H, a.S, 64))) return st;
  if ((st = tc_make_map(&mk, a.k, a.ks, a.B, a.H, a.S, 64))) return st;
  if ((st = tc_make_map(&mv, a.v, a.vs, a.B, a.H, a.S, 64))) return st;
  if ((st = tc_make_map(&mq128, a.q, a.qs, a.B, a.H, a.S, 128))) return st;
  if ((st = tc_make_map(&mdo128, a.dout, a.os, a.B, a.H, a.S, 128))) return st;
  if ((st = tc_make_map(&mk128, a.k, a.ks, a.B, a.H, a.S, 128))) return st;
  if ((st = tc_make_map(&mv128, a.v, a.vs, a.B, a.H, a.S, 128))) return st;

  int dev = 0;
  XSAKE_CUDA_TRY(cudaGetDevice(&dev));
  XSAKE_REQUIRE(dev < kMaxDev, XSAKE_EUNSUPPORTED, "device ordinal %d", dev);
  std::call_once(g_attr_once[dev], [dev] {
    g_attr_err[dev] =
        cudaFuncSetAttribute(tc_bwd_dkdv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kKvSmemBytes);
    if (g_attr_err[dev] == cudaSuccess)
      g_attr_err[dev] =
          cudaFuncSetAttribute(tc_bwd_dq_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kQSmemBytes);
  });
  XSAKE_REQUIRE(g_attr_err[dev] == cudaSuccess, XSAKE_ECUDA, "cudaFuncSetAttribute: %s",
                cudaGetErrorString(g_attr_err[dev]));

  XSAKE_CUDA_TRY(cudaMemsetAsync(counters, 0, 2 * sizeof(int), s));
  const int64_t nrows = bh * a.S;
  tc_bwd_prep_kernel<<<(unsigned)((nrows + 31) / 32), 256, 0, s>>>(a, nlse2, bias);
  if ((st = check_launch("tc_bwd_prep_kernel"))) return st;
  tc_ucol_kernel<<<(unsigned)bh, 64, 0, s>>>(a);
  if ((st = check_launch("tc_ucol_kernel"))) return st;

  BwdParams p;
  p.a = a;
  p.scale_log2 = a.scale * kLog2e;
  p.nlse2 = nlse2;
  p.bias = bias;
  p.counter = counters;
  const int grid = std::max(1, std::min(a.L.nitems, 2 * di.sm_count));
  tc_bwd_dkdv_kernel<<<grid, kThreads, kKvSmemBytes, s>>>(mk128, mv128, mq, mdo, p);
  if ((st = check_launch("tc_bwd_dkdv_kernel"))) return st;
  tc_bwd_dq_kernel<<<grid, kThreads, kQSmemBytes, s>>>(mq128, mdo128, mk, mv, p);
  return check_launch("tc_bwd_dq_kernel");
}

}  // namespace xsake
