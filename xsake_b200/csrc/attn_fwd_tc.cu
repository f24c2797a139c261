// HADS block-sparse attention forward on the sm_100a tensor cores (bf16 in, fp32 softmax
// statistics), head_dim 64, block sizes that are multiples of 64.
//
// Replaces _sparse_attn_fwd_kernel / sparse_attention_pallas
// (kernels/pallas/sparse_attention.py:96-156, :161-252).  Differences by design: only the
// active kv chunks of the compiled plan are visited (the reference loops over every block and
// discards masked ones, :147-153), the token-level causal mask is applied on diagonal chunks
// (the Pallas kernel ignores `causal`, the reference CPU path applies it, :79-81), and lse is
// returned.
//
// Each CTA (one per SM, persistent) runs two independent tile workers that share only the SM:
// each takes its own work items (128 query rows: in the query-chunk pairing the 64-row chunks
// 2t, 2t+1 of one (b, h), in the unit pairing one chunk of two units) from a global counter,
// longest first, and walks the ascending list of 64-key chunks the tile attends
// through its own 5-stage K/V ring (TMA, SWIZZLE_128B).  Two workers rather than one 256-row
// item over a merged chunk list: a merged walk made each tile's MMA warp wait on and release the
// other tile's chunks and kept the two softmax groups in lock-step (their exponential phases
// collided on MUFU, their waits left it idle together); independent workers drift apart.
// Chunks two neighbouring tiles share are read from L2 once per tile (K/V of a (b, h) is 1 MB
// and stays in L2).  Per tile and chunk: S = Q K^T (tcgen05, M=128 N=64
// K=64, fp32 in TMEM), softmax by one thread per query row straight out of TMEM, P (bf16)
// written back into TMEM over the first 32 columns of the scores it came from, O += P V
// (tcgen05 with A read from TMEM, fp32 accumulator resident in TMEM).  Keeping P out of shared
// memory matters: an M=128 N=64 K=16 MMA with both operands in shared memory reads 6 KB of it
// and is bound by shared-memory bandwidth (~50 cycles); with A in TMEM it reads 2 KB and runs at
// the tensor rate (~35 cycles), and the P stores and their proxy fence disappear.
// Roles (384 threads):
//   warps 0-3   softmax + epilogue of tile worker 0 (thread i owns row i = TMEM lane i)
//   warps 4-7   softmax + epilogue of tile worker 1
//   warps 8,9   scheduler + TMA producer of workers 0, 1: take items from the global counter,
//               publish them through a 2-slot ring, load Q (double-buffered) and K/V
//   warps 10,11 MMA issuers of workers 0, 1 (one elected lane each): QK of chunk i is queued
//               before PV of chunk i-2; a ring stage is released by the PV that read it
// TMEM: 512 columns; per tile (at 256*tile) three S buffers [0,64) [64,128) [128,192) so QK
// runs two chunks ahead of the softmax, and O at [192,256).  P of chunk s lives in S buffer s%3;
// the MMA warp issues QK of chunk s+3 (which overwrites it) only after PV of chunk s, and one
// thread's MMAs execute in issue order.
// The running max is only moved when it grows by more than 2^8 (rescaling O in TMEM is then
// rare); exp2 runs on MUFU for 3/4 of the elements and on a cubic polynomial for the rest.
//
// Two pairings share this structure (tile_roles and pair_roles, one kernel, tc_fwd_kernel, which
// runs the one the compiled plan names in its header word H_FWD_PAIR).  tile_roles pairs query
// chunks 2t, 2t+1 of one (b, h).  pair_roles pairs the same query chunk of two (b, h) units that
// share a mask (a mask broadcast over the batch or the heads, the usual HADS case); the plan
// compiler picks it when such units exist and the query-chunk pairing would leave more than 12%
// of its 64-row halves masked out (see the comment above PItem).
#include "attn_common.cuh"
#include "sm100.cuh"

#include <cudaTypedefs.h>
#include <algorithm>
#include <mutex>

XSAKE_DEFINE_DEVICE_ERROR(tcfwd)

namespace xsake {
namespace {

using namespace sm100;

constexpr int kStages = 5;                            // K/V ring stages per tile worker
constexpr int kQSlots = 2;                            // Q buffers per tile worker
constexpr uint32_t kPvLag = 3;                        // PV(s - kPvLag) is issued with QK(s)
constexpr int kThreads = 384;
constexpr int kQBytes = 128 * 64 * 2;
constexpr int kKBytes = 64 * 64 * 2;
constexpr int kStageBytes = 2 * kKBytes;
constexpr int kOffQ = 0;                              // [2 tiles][kQSlots]
constexpr int kOffKV = kOffQ + 2 * kQSlots * kQBytes;  // [2 tiles][kStages] K then V
constexpr int kOffBar = kOffKV + 2 * kStages * kStageBytes;

struct Bars {
  uint64_t item_full[2][2], item_empty[2][2];   // [tile][slot]
  uint64_t q_full[2][2], q_empty[2][2];
  uint64_t kv_full[2][kStages], kv_empty[2][kStages];
  uint64_t s_full[2][3];                 // [tile][S buffer]
  uint64_t p_full[2][3];                 // [tile][S buffer holding P]
  uint64_t o_done[2][2];                 // [tile][PV parity]
  uint64_t o_free[2];
  uint64_t ep_bar[2];                    // [tile]: the softmax warpgroup's split-merge rendezvous
  uint64_t drain;
};
constexpr int kOffMisc = kOffBar + (int)sizeof(Bars);
constexpr int kSmemBytes = kOffMisc + 64 + 1024;      // + alignment slack
static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kIdescQK = idesc_bf16(128, 64, false);
constexpr uint32_t kIdescPV = idesc_bf16(128, 64, true);
constexpr float kRescaleThreshold = 8.0f;             // log2 units
constexpr int kItemReaders = 1 + 128;                 // the tile's MMA warp + its softmax warpgroup

struct TcParams {
  AttnArgs a;
  float scale_log2;
  int o_rows_32b;     // output rows start on 32-byte boundaries (256-bit stores)
  int* counter;       // work-item counter, zeroed by the host before the launch
  int* grp_counter;   // [kSplitSlots] pieces finished per split group, zeroed with the counter
  float* parts;       // [kSplitSlots] partial slots of split pieces (kSlotFloats each)
};

__device__ __forceinline__ void fail(volatile int* abort, int detail) {
  if (atomicExch((int*)abort, 1) == 0) record_device_error(DEV_ERR_TIMEOUT, detail);
}


// Mean over all S rows of V[b, h] for the rare fully-masked rows; one warp, no block sync.
__device__ void warp_mean_v(const AttnArgs& a, int b, int h, float2& mine) {
  const int lane = threadIdx.x & 31;
  const __nv_bfloat16* v = reinterpret_cast<const __nv_bfloat16*>(a.v) + b * a.vs[0] + h * a.vs[1];
  float s0 = 0.f, s1 = 0.f;
  for (int r = 0; r < a.S; ++r) {
    const __nv_bfloat162 x = reinterpret_cast<const __nv_bfloat162*>(v + (int64_t)r * a.vs[2])[lane];
    s0 += __bfloat162float(x.x);
    s1 += __bfloat162float(x.y);
  }
  mine = make_float2(s0 / a.S, s1 / a.S);
}

// Entry `idx` of the plan's forward work table (two 16-byte loads).
__device__ __forceinline__ FWork load_work(const AttnArgs& a, int idx) {
  const int4* w = reinterpret_cast<const int4*>(a.plan + a.L.f_work_off) + 2 * (int64_t)idx;
  const int4 x = w[0], y = w[1];
  FWork f;
  f.u0 = x.x; f.u1 = x.y; f.q = x.z; f.lo = x.w;
  f.hi = y.x; f.parts = y.y; f.grp = y.z; f.slot = y.w;
  return f;
}

struct Item {
  int b, h, u, e0, n;
};

// The softmax warps hold a work entry spread over lanes 0-7 (lane i: word i of FWork), one
// register a thread, and shuffle fields out where they are used.
__device__ __forceinline__ int32_t work_lanes(const AttnArgs& a, int idx) {
  const int lane = threadIdx.x & 31;
  return lane < 8 ? a.plan[a.L.f_work_off + 8 * (int64_t)idx + lane] : 0;
}
__device__ __forceinline__ int32_t work_word(int32_t held, int i) { return __shfl_sync(0xffffffffu, held, i); }


__device__ __forceinline__ Item decode(const AttnArgs& a, int idx) {
  const FWork w = load_work(a, idx);
  Item it;
  it.u = w.q;
  it.b = w.u0 / a.H;
  it.h = w.u0 % a.H;
  it.e0 = w.lo;
  it.n = w.hi - w.lo;
  return it;
}

// Split pieces.  A piece of a split work item leaves its rows' unnormalised O, running max
// (log2 units) and row sum in its partial slot ([16][128][4] floats of O, then m[128], l[128]);
// the worker's 128 softmax threads meet on ep_bar (bounded waits), one of them counts the piece
// done, and the piece that completes its group merges every slot of the group in piece order,
// so the result does not depend on which piece finished last.
constexpr int kSlotFloats = 128 * 64 + 2 * 128;

// Returns true when this piece was the group's last and m, l, o now hold the merged row.
__device__ __forceinline__ bool split_finish(const TcParams& p, int grp, int part, int nparts, int slot0, int srow,
                                             uint64_t* ep_bar, uint32_t& ep_phase, volatile int* flag, float& m,
                                             float& l, float (&o)[64], volatile int* abort, bool& ok) {
  float* mine = p.parts + (int64_t)(slot0 + part) * kSlotFloats;
  float4* ob = reinterpret_cast<float4*>(mine);
#pragma unroll
  for (int k = 0; k < 16; ++k) ob[k * 128 + srow] = make_float4(o[4 * k], o[4 * k + 1], o[4 * k + 2], o[4 * k + 3]);
  mine[128 * 64 + srow] = m;
  mine[128 * 64 + 128 + srow] = l;
  // The warpgroup's stores are ordered before one thread's gpu-scope release by the CTA-scope
  // rendezvous (the pattern of a grid barrier: only the counting thread fences); the counting
  // thread's acquire orders the merge's loads after the other pieces' stores, and the second
  // rendezvous hands that order to the warpgroup.
  mbar_arrive(ep_bar);
  if (!warp_mbar_wait(ep_bar, ep_phase & 1, abort)) { ok = false; return false; }
  ++ep_phase;
  if (srow == 0) {
    int old;
    asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], 1;" : "=r"(old) : "l"(p.grp_counter + grp) : "memory");
    *flag = old == nparts - 1;
  }
  mbar_arrive(ep_bar);
  if (!warp_mbar_wait(ep_bar, ep_phase & 1, abort)) { ok = false; return false; }
  ++ep_phase;
  if (!*flag) return false;
  float M = -INFINITY;
  for (int q = 0; q < nparts; ++q) {
    const float* pq = p.parts + (int64_t)(slot0 + q) * kSlotFloats;
    if (__ldcg(pq + 128 * 64 + 128 + srow) > 0.f) M = fmaxf(M, __ldcg(pq + 128 * 64 + srow));
  }
  float lt = 0.f;
#pragma unroll
  for (int c = 0; c < 64; ++c) o[c] = 0.f;
  for (int q = 0; q < nparts; ++q) {
    const float* pq = p.parts + (int64_t)(slot0 + q) * kSlotFloats;
    const float lq = __ldcg(pq + 128 * 64 + 128 + srow);
    if (!(lq > 0.f)) continue;
    const float f = ex2(__ldcg(pq + 128 * 64 + srow) - M);
    lt += lq * f;
    const float4* oq = reinterpret_cast<const float4*>(pq);
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      const float4 v = __ldcg(oq + k * 128 + srow);
      o[4 * k] += v.x * f;
      o[4 * k + 1] += v.y * f;
      o[4 * k + 2] += v.z * f;
      o[4 * k + 3] += v.w * f;
    }
  }
  m = M;
  l = lt;
  return true;
}

// The row's O accumulator (64 fp32 columns at TMEM column `taddr`) into registers.
__device__ __forceinline__ void load_o_row(uint32_t taddr, float (&o)[64]) {
  uint32_t r[64];
  XSAKE_TMEM_LD32(taddr, r);
  XSAKE_TMEM_LD32(taddr + 32, (r + 32));
  XSAKE_TMEM_WAIT_LD32(r);
  XSAKE_TMEM_WAIT_LD32((r + 32));
#pragma unroll
  for (int j = 0; j < 64; ++j) o[j] = __uint_as_float(r[j]);
}

// One bf16 output row: o * inv, eight 16-byte stores.
__device__ __forceinline__ void store_o_row(uint4* orow_g, const float (&o)[64], float inv, bool v8) {
  // Four 32-byte stores (whole sectors) when the row starts on a 32-byte boundary: the epilogue's
  // row-per-thread stores are the largest item-boundary cost of the softmax warps (A/B: 121.6-121.9
  // vs 122.5-124.1 us on config 3, identical outputs).
  if (v8) {
#pragma unroll
    for (int cc = 0; cc < 4; ++cc) {
      uint32_t wv[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        __nv_bfloat162 pb = __floats2bfloat162_rn(o[16 * cc + 2 * q] * inv, o[16 * cc + 2 * q + 1] * inv);
        wv[q] = *reinterpret_cast<uint32_t*>(&pb);
      }
      asm volatile("st.global.v8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"l"(orow_g + 2 * cc), "r"(wv[0]), "r"(wv[1]),
                   "r"(wv[2]), "r"(wv[3]), "r"(wv[4]), "r"(wv[5]), "r"(wv[6]), "r"(wv[7])
                   : "memory");
    }
    return;
  }
#pragma unroll
  for (int cc = 0; cc < 8; ++cc) {
    uint32_t wv[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      __nv_bfloat162 pb = __floats2bfloat162_rn(o[8 * cc + 2 * q] * inv, o[8 * cc + 2 * q + 1] * inv);
      wv[q] = *reinterpret_cast<uint32_t*>(&pb);
    }
    orow_g[cc] = make_uint4(wv[0], wv[1], wv[2], wv[3]);
  }
}

// Entry i of an item's list for a whole warp.  The list is read 32 entries at a time into lane
// registers (lane j holds entry base + j) and handed out with a shuffle, so walking the list
// costs no dependent global load per entry.  i must be visited in increasing order.
template <class W>
__device__ __forceinline__ int32_t entry_at(const int32_t* entries, const W& w, int i, int32_t& held,
                                            int& base) {
  if (i >= base + 32) {
    base = i & ~31;
    const int j = base + (int)(threadIdx.x & 31);
    held = j < w.n ? entries[w.e0 + j] : 0;
  }
  return __shfl_sync(0xffffffffu, held, i - base);
}

// State the role functions share: set up once per CTA by tc_fwd_kernel.
struct FwdCtx {
  uint8_t* smem;
  Bars* bars;
  volatile int* abort;
  volatile int* item_slots;   // [tile worker][slot]
  volatile int* ep_flag;      // [tile worker]: this piece completed its split group
  uint32_t tmem;
  const int32_t* entries;
};

// Row max of 64 raw scores: a depth-4 tree of 3-input maxes.
__device__ __forceinline__ float rowmax64(const float* x) {
  float t1[22];
#pragma unroll
  for (int j = 0; j < 21; ++j) t1[j] = max3(x[3 * j], x[3 * j + 1], x[3 * j + 2]);
  t1[21] = x[63];
  float t2[8];
#pragma unroll
  for (int j = 0; j < 7; ++j) t2[j] = max3(t1[3 * j], t1[3 * j + 1], t1[3 * j + 2]);
  t2[7] = t1[21];
  return fmaxf(max3(t2[0], t2[1], t2[2]), max3(t2[3], t2[4], fmaxf(t2[5], fmaxf(t2[6], t2[7]))));
}

// Output rows of a query-chunk-pairing item (tile_roles) once the row's O (64 fp32),
// running max m (log2 units) and sum l are in registers: the split merge (a piece that leaves it
// to another piece writes nothing), O / l in bf16, the uniform attention of rows with no live
// score, and lse.  The whole warp calls it.
__device__ __forceinline__ void tile_output(const TcParams& p, const FwdCtx& c, int X, int row, int32_t wk, float m,
                                            float l, float (&o)[64], uint32_t& ep_phase, bool& ok) {
  const AttnArgs& a = p.a;
  const int grp = work_word(wk, 6), parts = work_word(wk, 5);
  if (grp >= 0 && !split_finish(p, grp, parts >> 8, parts & 0xff, work_word(wk, 7), row, &c.bars->ep_bar[X],
                                ep_phase, c.ep_flag + X, m, l, o, c.abort, ok))
    return;   // another piece of this item merges the rows (or a wait failed: ok is false)
  const int u0 = work_word(wk, 0);
  const Item we{u0 / a.H, u0 % a.H, work_word(wk, 2), 0, 0};
  const int tok = 128 * we.u + row;
  const bool valid = tok < a.S;
  const bool empty = valid && !(l > 0.f);
  uint4* orow_g = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(a.o) + we.b * a.os[0] +
                                           we.h * a.os[1] + (int64_t)(valid ? tok : 0) * a.os[2]);
  if (valid && !empty) store_o_row(orow_g, o, 1.f / l, p.o_rows_32b);
  if (__any_sync(0xffffffffu, empty)) {
    // Rows with no live score: the reference's finfo.min fill makes them attend uniformly.
    float2 mine;
    warp_mean_v(a, we.b, we.h, mine);
#pragma unroll
    for (int cc = 0; cc < 8; ++cc) {
      uint32_t wv[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int src = 4 * cc + q;   // column pair index 0..31
        __nv_bfloat162 pb = __floats2bfloat162_rn(__shfl_sync(0xffffffffu, mine.x, src),
                                                  __shfl_sync(0xffffffffu, mine.y, src));
        wv[q] = *reinterpret_cast<uint32_t*>(&pb);
      }
      if (empty) orow_g[cc] = make_uint4(wv[0], wv[1], wv[2], wv[3]);
    }
  }
  if (valid) a.lse[(int64_t)(we.b * a.H + we.h) * a.S + tok] = empty ? kMaskFill : (m + __log2f(l)) * kLn2;
}

// Roles of the query-chunk pairing: a work item is query chunks 2t, 2t+1 of one (b, h).
__device__ __forceinline__ void tile_roles(const CUtensorMap& tmQ, const CUtensorMap& tmK,
                                           const CUtensorMap& tmV, const TcParams& p, const FwdCtx& c) {
  uint8_t* smem = c.smem;
  Bars* bars = c.bars;
  volatile int* abort = c.abort;
  volatile int* item_slots = c.item_slots;
  const uint32_t tmem = c.tmem;
  const int32_t* entries = c.entries;
  const AttnArgs& a = p.a;
  const PlanLayout& L = a.L;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nwork = a.plan[H_F_WORK];
  if (warp == 8 || warp == 9) {
    // ------------------------------------------------------------------ scheduler + TMA
    // One warp per tile (X = warp - 8); the whole warp runs the (uniform) control flow, one
    // elected lane issues.
    const int X = warp - 8;
    volatile int* item_slot = item_slots + 2 * X;
    uint8_t* kv0 = smem + kOffKV + X * kStages * kStageBytes;
    uint32_t it = 0, qk = 0;
    bool ok = true;
    for (uint32_t k = 0; ok; ++k) {
      const int slot = k & 1;
      if (!warp_mbar_wait(&bars->item_empty[X][slot], ((k >> 1) & 1) ^ 1, abort)) { ok = false; break; }
      int idx = 0;
      if (lane == 0) idx = *abort ? nwork : atomicAdd(p.counter, 1);
      idx = __shfl_sync(0xffffffffu, idx, 0);
      const int item = idx < nwork ? idx : -1;
      if (elect_one()) {
        item_slot[slot] = item;
        mbar_arrive(&bars->item_full[X][slot]);
      }
      __syncwarp();
      if (item < 0) break;
      const Item w = decode(a, item);
      if (w.n == 0) continue;
      const int qs = qk % kQSlots;
      if (!warp_mbar_wait(&bars->q_empty[X][qs], ((qk / kQSlots) & 1) ^ 1, abort)) { ok = false; break; }
      if (elect_one()) {
        mbar_arrive_expect_tx(&bars->q_full[X][qs], kQBytes);
        uint8_t* qbuf = smem + kOffQ + (kQSlots * X + qs) * kQBytes;   // two 64-row boxes
          tma_load_4d(qbuf, &tmQ, &bars->q_full[X][qs], 0, 128 * w.u, w.h, w.b);
          tma_load_4d(qbuf + kQBytes / 2, &tmQ, &bars->q_full[X][qs], 0, 128 * w.u + 64, w.h, w.b);
      }
      __syncwarp();
      ++qk;
      int32_t held = 0;
      int base = -32;
      for (int i = 0; i < w.n; ++i, ++it) {
        const int c = entry_at(entries, w, i, held, base) & kEntryIdxMask;
        const int st = it % kStages;
        if (!warp_mbar_wait(&bars->kv_empty[X][st], ((it / kStages) & 1) ^ 1, abort)) { ok = false; break; }
        if (elect_one()) {
          uint8_t* kbuf = kv0 + st * kStageBytes;
          mbar_arrive_expect_tx(&bars->kv_full[X][st], kStageBytes);
          tma_load_4d(kbuf, &tmK, &bars->kv_full[X][st], 0, 64 * c, w.h, w.b);
          tma_load_4d(kbuf + kKBytes, &tmV, &bars->kv_full[X][st], 0, 64 * c, w.h, w.b);
        }
        __syncwarp();
      }
    }
    if (!ok && lane == 0) {
      fail(abort, 1);
      // Give copies in flight a bounded chance to land before the CTA exits.
      for (int s = 0; s < kStages; ++s) {
        const uint64_t t0 = global_timer_ns();
        while (!mbar_try_wait(&bars->kv_full[X][s], 0) && !mbar_try_wait(&bars->kv_full[X][s], 1) &&
               global_timer_ns() - t0 < 1000000ull) {
        }
      }
    }
  } else if (warp == 10 || warp == 11) {
    // ------------------------------------------------------------------ MMA issuers
    // One warp per tile worker (X = warp - 10).
    // The whole warp runs the (uniform) control flow; one elected lane issues.  The entries
    // of the item are visited in order (the plan lists only chunks the tile attends; an entry
    // without an active flag would be released unused, after its load landed).  QK of step s
    // goes into S buffer s%3 once PV(s-3) has been issued (which implies the softmax has read
    // S(s-3)); PV(s-2) is issued right after QK(s), the item's last ones at its end.
    const int X = warp - 10;
    volatile int* item_slot = item_slots + 2 * X;
    const int32_t f_tile = kEntryFlags;
    const uint32_t tcol = tmem + 256 * X;
    const uint64_t kdesc0 = sw128_desc(smem_u32(smem + kOffKV + X * kStages * kStageBytes), 16, 1024);
    uint32_t it = 0, qk = 0, steps = 0, pvs = 0, titems = 0, item_first = 0;
    int pst0 = 0, pst1 = 0, pst2 = 0;   // ring stage of the step in S buffer 0, 1, 2 (registers)
    auto pstage = [&](uint32_t b) { return b == 0 ? pst0 : (b == 1 ? pst1 : pst2); };
    bool ok = true;
    auto issue_pv = [&]() -> bool {
      const uint32_t s = pvs, pb = s & 1, sbuf = s % 3;
      if (!warp_mbar_wait(&bars->p_full[X][sbuf], (s / 3) & 1, abort)) return false;
      const bool first = (s == item_first);
      if (first && titems > 0 && !warp_mbar_wait(&bars->o_free[X], (titems - 1) & 1, abort)) return false;
      tc_fence_after();
      const int st = pstage(sbuf);
      if (elect_one()) {
        const uint64_t vdesc = kdesc0 + (uint64_t)((st * kStageBytes + kKBytes) >> 4);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)   // O += P V, P = 16 keys per 8 TMEM columns
          mma_bf16_ts(tcol + 192, tcol + 64 * sbuf + 8 * kk, vdesc + (uint64_t)((2048 * kk) >> 4), kIdescPV,
                      (first && kk == 0) ? 0u : 1u);
        mma_commit(&bars->o_done[X][pb]);
        mma_commit(&bars->kv_empty[X][st]);
      }
      __syncwarp();
      ++pvs;
      return true;
    };
    for (uint32_t k = 0; ok; ++k) {
      const int slot = k & 1;
      if (!warp_mbar_wait(&bars->item_full[X][slot], (k >> 1) & 1, abort)) { ok = false; break; }
      const int item = item_slot[slot];
      __syncwarp();
      if (elect_one()) mbar_arrive(&bars->item_empty[X][slot]);
      __syncwarp();
      if (item < 0) break;
      const Item w = decode(a, item);
      if (w.n == 0) continue;
      const int qs = qk % kQSlots;
      if (!warp_mbar_wait(&bars->q_full[X][qs], (qk / kQSlots) & 1, abort)) { ok = false; break; }
      ++qk;
      const uint64_t qdesc = sw128_desc(smem_u32(smem + kOffQ + (kQSlots * X + qs) * kQBytes), 16, 1024);
      item_first = steps;
      int last_used = -1;
      for (int b0 = 0; b0 < w.n; b0 += 32) {
        const int j = b0 + lane;
        const uint32_t own = __ballot_sync(0xffffffffu, j < w.n && (entries[w.e0 + j] & f_tile) != 0);
        if (own) last_used = b0 + 31 - __clz(own);
      }
      int32_t held = 0;
      int base = -32;
      for (int i = 0; i < w.n && ok; ++i, ++it) {
        const int32_t e = entry_at(entries, w, i, held, base);
        const int st = it % kStages;
        if (!(e & f_tile)) {
          // Pending PVs hold ring stages: issue them before waiting on an entry that is not used.
          while (ok && pvs < steps) ok = issue_pv();
          if (!ok || !warp_mbar_wait(&bars->kv_full[X][st], (it / kStages) & 1, abort)) { ok = false; break; }
          if (elect_one()) mbar_arrive(&bars->kv_empty[X][st]);
          __syncwarp();
          continue;
        }
        // One batch per step: PV(steps - kPvLag) of this item, then QK(steps) (which needs
        // PV(steps - 3) issued, so kPvLag <= 3), after one combined wait for both operands.
        while (ok && pvs + kPvLag < steps) ok = issue_pv();
        if (!ok) break;
        const bool pv_now = pvs + kPvLag == steps;
        const uint32_t ps = pvs, psb = ps % 3;
        const bool pv_first = pv_now && ps == item_first;
        if (pv_first && titems > 0 && !warp_mbar_wait(&bars->o_free[X], (titems - 1) & 1, abort)) { ok = false; break; }
        if (!warp_mbar_wait2(&bars->kv_full[X][st], (it / kStages) & 1, &bars->p_full[X][psb], (ps / 3) & 1,
                             pv_now, abort)) { ok = false; break; }
        const uint32_t sb = steps % 3;
        tc_fence_after();
        if (elect_one()) {
          if (pv_now) {
            const int pst = pstage(psb);
            const uint64_t vdesc = kdesc0 + (uint64_t)((pst * kStageBytes + kKBytes) >> 4);
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              mma_bf16_ts(tcol + 192, tcol + 64 * psb + 8 * kk, vdesc + (uint64_t)((2048 * kk) >> 4), kIdescPV,
                          (pv_first && kk == 0) ? 0u : 1u);
            mma_commit(&bars->o_done[X][ps & 1]);
            mma_commit(&bars->kv_empty[X][pst]);
          }
          const uint64_t kdesc = kdesc0 + (uint64_t)((st * kStageBytes) >> 4);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            mma_bf16_ss(tcol + 64 * sb, qdesc + 2 * kk, kdesc + 2 * kk, kIdescQK, kk > 0 ? 1u : 0u);
          mma_commit(&bars->s_full[X][sb]);
          if (i == last_used) mma_commit(&bars->q_empty[X][qs]);
        }
        __syncwarp();
        if (pv_now) ++pvs;
        pst0 = sb == 0 ? st : pst0;
        pst1 = sb == 1 ? st : pst1;
        pst2 = sb == 2 ? st : pst2;
        ++steps;
      }
      if (!ok) break;
      while (ok && pvs < steps) ok = issue_pv();
      if (!ok) break;
      if (last_used < 0) {           // this tile had nothing in the item: release its Q share
        if (elect_one()) mbar_arrive(&bars->q_empty[X][qs]);
        __syncwarp();
      }
      if (steps > item_first) ++titems;
    }
    if (!ok && lane == 0) fail(abort, 3);
    // Drain: no MMA may be in flight when TMEM is released.
    if (elect_one()) mma_commit(&bars->drain);
    __syncwarp();
    if (lane == 0) {
      const uint64_t t0 = global_timer_ns();
      while (!mbar_try_wait(&bars->drain, 0) && global_timer_ns() - t0 < kWaitLimitNs) {
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------------ softmax + epilogue
    const int X = warp >> 2;                 // tile
    const int row = threadIdx.x & 127;       // TMEM lane
    const int half = row >> 6;
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    const uint32_t tcol = tmem + 256 * X;
    volatile int* item_slot = item_slots + 2 * X;
    const int32_t f_tile = kEntryFlags;
    const int32_t f_active = half ? kFlagActive1 : kFlagActive0;
    const int32_t f_diag = half ? kFlagDiag1 : kFlagDiag0;
    const int diag_lim = row & 63;
    uint64_t* s_full = bars->s_full[X];
    uint64_t* p_full = bars->p_full[X];
    uint64_t* o_done = bars->o_done[X];
    uint64_t* o_free = &bars->o_free[X];
    uint32_t it = 0, sb_c = 0, ph_c = 0;   // step count, its S buffer (it % 3) and phase ((it / 3) & 1)
    bool s_ready = false;                  // S of step `it` already seen complete by every lane
    uint32_t ep_phase = 0;                 // uses of ep_bar[X]
    bool ok = true;
    for (uint32_t k = 0; ok; ++k) {
      const int slot = k & 1;
      if (!warp_mbar_wait(&bars->item_full[X][slot], (k >> 1) & 1, abort)) { ok = false; break; }
      const int item = item_slot[slot];
      mbar_arrive(&bars->item_empty[X][slot]);
      if (item < 0) break;
      const int32_t wk = work_lanes(a, item);
      const int we0 = work_word(wk, 3), wn = work_word(wk, 4) - we0;
      float m = -INFINITY, l = 0.f;
      int nsteps = 0;
      // The item's entries, 32 at a time: a ballot marks them and a shuffle hands each one out.
      for (int b0 = 0; b0 < wn && ok; b0 += 32) {
        const int32_t eb = b0 + lane < wn ? entries[we0 + b0 + lane] : 0;
        uint32_t own = __ballot_sync(0xffffffffu, (eb & f_tile) != 0);
        while (own) {
          const int32_t e = __shfl_sync(0xffffffffu, eb, __ffs(own) - 1);
          own &= own - 1;
          ++nsteps;
          const uint32_t sb = sb_c;
          if (!s_ready && !warp_mbar_wait(&s_full[sb], ph_c, abort)) { ok = false; break; }
          tc_fence_after();
          uint32_t sr[64];
          XSAKE_TMEM_LD32(tcol + lane_base + 64 * sb, sr);
          XSAKE_TMEM_LD32(tcol + lane_base + 64 * sb + 32, (sr + 32));
          // Probe the next step's S while the load is in flight (non-blocking; the QKs run
          // ahead, so it has usually landed): a complete phase seen by every lane saves the
          // next wait.  The probe has acquire semantics, like the wait it replaces.
          const bool next_done = mbar_test_wait(&s_full[sb_c == 2 ? 0 : sb_c + 1], sb_c == 2 ? ph_c ^ 1u : ph_c);
          XSAKE_TMEM_WAIT_LD32(sr);
          XSAKE_TMEM_WAIT_LD32((sr + 32));
          s_ready = __all_sync(0xffffffffu, next_done);
          uint32_t pk[32];
          if (e & f_active) {
            float* x = reinterpret_cast<float*>(sr);   // raw scores
            if (e & f_diag) {                          // warp-uniform: token-level causal cut
#pragma unroll
              for (int j = 0; j < 64; ++j)
                if (j > diag_lim) x[j] = -INFINITY;
            }
            const float mx = rowmax64(x) * p.scale_log2;   // log2 units (scale > 0)
            const bool need = (m != -INFINITY) && (mx > m + kRescaleThreshold);
            if (m == -INFINITY) m = mx;
            // TMEM loads/stores are warp-collective: the whole warp rescales when any row must.
            if (__any_sync(0xffffffffu, need)) {
              // O holds PV of earlier chunks: wait for the last one, then rescale in TMEM.
              if (!warp_mbar_wait(&o_done[(it - 1) & 1], ((it - 1) >> 1) & 1, abort)) { ok = false; break; }
              tc_fence_after();
              const float alpha = need ? ex2(m - mx) : 1.0f;
              uint32_t orow[32];
#pragma unroll
              for (int hcol = 0; hcol < 2; ++hcol) {
                XSAKE_TMEM_LD32(tcol + lane_base + 192 + 32 * hcol, orow);
                XSAKE_TMEM_WAIT_LD32(orow);
#pragma unroll
                for (int j = 0; j < 32; ++j) orow[j] = __float_as_uint(__uint_as_float(orow[j]) * alpha);
                XSAKE_TMEM_ST32(tcol + lane_base + 192 + 32 * hcol, orow);
              }
              tmem_wait_st();
              if (need) {
                l *= alpha;
                m = mx;
              }
            }
            const float msub = (m == -INFINITY) ? 0.f : m;   // no live score yet: every x is -inf
            // p = 2^(s*scale*log2e - m): one packed FMA per pair; 2 of every 8 pairs go through
            // the polynomial exp2 on the FMA/ALU pipes, the rest through MUFU ex2.
            const uint64_t cc = pk2(p.scale_log2, p.scale_log2), nm = pk2(-msub, -msub);
            uint64_t acc[4] = {0ull, 0ull, 0ull, 0ull};
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              float x0, x1, p0, p1;
              upk2(fma2(pk2(x[2 * j], x[2 * j + 1]), cc, nm), x0, x1);
              if ((j & 7) < 2) {
                exp2_poly2(x0, x1, p0, p1);
              } else {
                p0 = ex2(x0);
                p1 = ex2(x1);
              }
              acc[j & 3] = add2(acc[j & 3], pk2(p0, p1));
              __nv_bfloat162 pb = __floats2bfloat162_rn(p0, p1);
              pk[j] = *reinterpret_cast<uint32_t*>(&pb);
            }
            float s0, s1;
            upk2(add2(add2(acc[0], acc[1]), add2(acc[2], acc[3])), s0, s1);
            l += s0 + s1;
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) pk[j] = 0u;
          }
          // P over the first 32 columns of the S buffer this thread has just read (its own row).
          XSAKE_TMEM_ST32(tcol + lane_base + 64 * sb, pk);
          tmem_wait_st();
          tc_fence_before();
          mbar_arrive(&p_full[sb]);
          ++it;
          if (++sb_c == 3) {
            sb_c = 0;
            ph_c ^= 1;
          }
        }
      }
      if (!ok) break;
      // ---------------------------------------------------------------- epilogue
      float o[64];
      if (nsteps > 0) {
        // PV(s) completes phase s/2 of o_done[s % 2].  A parity wait for PV(it-1) is only
        // unambiguous if that barrier's previous phase (PV(it-3)) has completed; the last S
        // buffer seen (QK(it-1)) only implies PV(it-4).  So wait for PV(it-2) first (its
        // previous phase, PV(it-4), is known complete), which implies PV(it-3), then PV(it-1).
        // (Inside the loop the rescale at step it is safe: QK(it) implies PV(it-3).)
        if (it >= 2 && !warp_mbar_wait(&o_done[(it - 2) & 1], ((it - 2) >> 1) & 1, abort)) { ok = false; break; }
        if (!warp_mbar_wait(&o_done[(it - 1) & 1], ((it - 1) >> 1) & 1, abort)) { ok = false; break; }
        tc_fence_after();
        load_o_row(tcol + lane_base + 192, o);
        tc_fence_before();
        mbar_arrive(o_free);
      } else {
#pragma unroll
        for (int j = 0; j < 64; ++j) o[j] = 0.f;
      }
      tile_output(p, c, X, row, wk, m, l, o, ep_phase, ok);
    }
    if (!ok) fail(abort, 4);
  }
}


// ---------------------------------------------------------------------------------------------
// Unit pairing.  A mask broadcast over the batch (or the heads) gives several (b, h)
// units the same chunk lists.  A work item of this pairing is one 64-row query chunk j of TWO
// such units u0, u1: every step is one 64-key chunk c that chunk j attends, computed for both
// units at once, so both halves of every step do useful work.  The query-chunk pairing walks
// the union of two chunks' lists instead; on HADS masks the two lists differ in their random
// long-range picks and 23% of its half-steps are masked out.  The price of this pairing is the
// M=64 MMAs (about the tensor time of M=128 ones for half the rows) and twice the K/V loads per
// step: measured, it wins at 67-80% useful half-steps (bigbird, HADS, local windows: 3-8%) and
// loses 7% on a dense causal mask (98.5%).
//
// The two units' scores and outputs are M=64 accumulators interleaved in TMEM: unit u0's row r
// sits in lane 32*(r/16) + r%16, unit u1's in the same lane + 16, so each softmax warp holds 16
// rows of each unit (lanes 0-15: u0, lanes 16-31: u1) and still owns one row per thread.  Per
// step and unit: S = Q K^T (tcgen05 M=64 N=64, A and B in shared memory), P written back over
// the first 32 columns of the unit's scores, O += P V (M=64, A read from the same TMEM lanes as
// the accumulator).  A ring slot holds one unit's K and V chunk; a step takes two consecutive
// slots (u0's, then u1's).  Roles, barriers, the scheduler, bounded waits and the softmax
// arithmetic are those of the query-chunk pairing.  Items are taken in descending j (longest lists first
// under a causal mask).  With an odd number of units per mask the last unit of each group runs
// alone: its partner lanes are masked out and its second slot is released without a load.
struct PItem {
  int b0, h0, b1, h1, j, e0, n;
  bool solo;
};

__device__ __forceinline__ PItem decode_pair(const AttnArgs& a, int idx) {
  const FWork w = load_work(a, idx);
  PItem it;
  it.j = w.q;
  it.solo = w.u1 < 0;
  const int u1 = it.solo ? w.u0 : w.u1;
  it.b0 = w.u0 / a.H;
  it.h0 = w.u0 % a.H;
  it.b1 = u1 / a.H;
  it.h1 = u1 % a.H;
  it.e0 = w.lo;
  it.n = w.hi - w.lo;
  return it;
}

// Number of entries of the list carrying flag f, and the index of the last one (-1 if none).
__device__ __forceinline__ int count_steps(const int32_t* entries, int e0, int n, int32_t f, int& last) {
  const int lane = threadIdx.x & 31;
  int cnt = 0;
  last = -1;
  for (int b0 = 0; b0 < n; b0 += 32) {
    const int j = b0 + lane;
    const uint32_t own = __ballot_sync(0xffffffffu, j < n && (entries[e0 + j] & f) != 0);
    cnt += __popc(own);
    if (own) last = b0 + 31 - __clz(own);
  }
  return cnt;
}

constexpr uint32_t kIdescQK64 = idesc_bf16(64, 64, false);
constexpr uint32_t kIdescPV64 = idesc_bf16(64, 64, true);
constexpr uint32_t kLane16 = 16u << 16;   // TMEM address of the partner unit's lanes
// PV lag of the unit pairing: 2 measured 1% faster than 3 there (one step less QK run-ahead,
// PV issued a step sooner); the query-chunk pairing keeps 3 (2 was 3% slower on a dense mask).
// QK(s) still follows PV(s-3) in issue order, so the S buffer it overwrites has been read.
constexpr uint32_t kPairPvLag = 2;
constexpr int kPairKStages = 2;           // K ring (both units' K chunks per stage), released by QK
constexpr int kPairVStages = 3;           // V ring, released by PV
static_assert(kPairKStages + kPairVStages <= kStages, "the pair rings reuse the K/V ring's shared memory");

// Roles of the unit pairing (see the comment above PItem).
__device__ __forceinline__ void pair_roles(const CUtensorMap& tmQ, const CUtensorMap& tmK,
                                           const CUtensorMap& tmV, const TcParams& p, const FwdCtx& c) {
  uint8_t* smem = c.smem;
  Bars* bars = c.bars;
  volatile int* abort = c.abort;
  volatile int* item_slots = c.item_slots;
  const uint32_t tmem = c.tmem;
  const int32_t* entries = c.entries;
  const AttnArgs& a = p.a;
  const PlanLayout& L = a.L;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nwork = a.plan[H_F_WORK];
  if (warp == 8 || warp == 9) {
    // ------------------------------------------------------------------ scheduler + TMA
    const int X = warp - 8;
    volatile int* item_slot = item_slots + 2 * X;
    uint8_t* kv0 = smem + kOffKV + X * kStages * kStageBytes;
    uint32_t it = 0, qk = 0;
    bool ok = true;
    for (uint32_t k = 0; ok; ++k) {
      const int slot = k & 1;
      if (!warp_mbar_wait(&bars->item_empty[X][slot], ((k >> 1) & 1) ^ 1, abort)) { ok = false; break; }
      int idx = 0;
      if (lane == 0) idx = *abort ? nwork : atomicAdd(p.counter, 1);
      idx = __shfl_sync(0xffffffffu, idx, 0);
      const int item = idx < nwork ? idx : -1;
      if (elect_one()) {
        item_slot[slot] = item;
        mbar_arrive(&bars->item_full[X][slot]);
      }
      __syncwarp();
      if (item < 0) break;
      const PItem w = decode_pair(a, item);
      const int32_t fa = (w.j & 1) ? kFlagActive1 : kFlagActive0;
      int last = -1;
      if (count_steps(entries, w.e0, w.n, fa, last) == 0) continue;
      const int qs = qk % kQSlots;
      if (!warp_mbar_wait(&bars->q_empty[X][qs], ((qk / kQSlots) & 1) ^ 1, abort)) { ok = false; break; }
      if (elect_one()) {
        uint8_t* qbuf = smem + kOffQ + (kQSlots * X + qs) * kQBytes;
        mbar_arrive_expect_tx(&bars->q_full[X][qs], w.solo ? kQBytes / 2 : kQBytes);
        tma_load_4d(qbuf, &tmQ, &bars->q_full[X][qs], 0, 64 * w.j, w.h0, w.b0);
        if (!w.solo) tma_load_4d(qbuf + kQBytes / 2, &tmQ, &bars->q_full[X][qs], 0, 64 * w.j, w.h1, w.b1);
      }
      __syncwarp();
      ++qk;
      // K of step s goes out before V of step s-1: V(s-1) waits for PV(s-4), which the MMA
      // warp issues only with QK(s-1), so K is never held up behind a V slot.
      const uint32_t bytes = w.solo ? kKBytes : 2 * kKBytes;
      auto load_pair = [&](const CUtensorMap* map, int bar, uint8_t* buf, int c) {
        if (elect_one()) {
          mbar_arrive_expect_tx(&bars->kv_full[X][bar], bytes);
          tma_load_4d(buf, map, &bars->kv_full[X][bar], 0, 64 * c, w.h0, w.b0);
          if (!w.solo) tma_load_4d(buf + kKBytes, map, &bars->kv_full[X][bar], 0, 64 * c, w.h1, w.b1);
        }
        __syncwarp();
      };
      auto load_v = [&](uint32_t s, int c) -> bool {
        const int vs = s % kPairVStages;
        if (!warp_mbar_wait(&bars->kv_empty[X][kPairKStages + vs], ((s / kPairVStages) & 1) ^ 1, abort))
          return false;
        load_pair(&tmV, kPairKStages + vs, kv0 + (kPairKStages + vs) * kStageBytes, c);
        return true;
      };
      int32_t held = 0;
      int base = -32, pend_c = -1;
      for (int i = 0; i < w.n && ok; ++i) {
        const int32_t e = entry_at(entries, w, i, held, base);
        if (!(e & fa)) continue;
        const int c = e & kEntryIdxMask;
        const int ks = it % kPairKStages;
        if (!warp_mbar_wait(&bars->kv_empty[X][ks], ((it / kPairKStages) & 1) ^ 1, abort)) { ok = false; break; }
        load_pair(&tmK, ks, kv0 + ks * kStageBytes, c);
        if (pend_c >= 0 && !load_v(it - 1, pend_c)) { ok = false; break; }
        pend_c = c;
        ++it;
      }
      if (ok && pend_c >= 0 && !load_v(it - 1, pend_c)) ok = false;
    }
    if (!ok && lane == 0) {
      fail(abort, 1);
      for (int s = 0; s < kStages; ++s) {
        const uint64_t t0 = global_timer_ns();
        while (!mbar_try_wait(&bars->kv_full[X][s], 0) && !mbar_try_wait(&bars->kv_full[X][s], 1) &&
               global_timer_ns() - t0 < 1000000ull) {
        }
      }
    }
  } else if (warp == 10 || warp == 11) {
    // ------------------------------------------------------------------ MMA issuers
    // Per step: one combined wait (K(s) landed; P(s-2) written and V(s-2) landed), then PV(s-2)
    // and QK(s) for both units.  This warp's loop is on the softmax's critical path (it shares its
    // sub-partition with two busy softmax warps), so it carries as few instructions as possible:
    // one combined wait and no walk of the entry list (A/B: 117.1 vs 128.1 us).
    const int X = warp - 10;
    volatile int* item_slot = item_slots + 2 * X;
    const uint32_t tcol = tmem + 256 * X;
    const uint64_t kdesc0 = sw128_desc(smem_u32(smem + kOffKV + X * kStages * kStageBytes), 16, 1024);
    uint32_t qk = 0, steps = 0, pvs = 0, titems = 0, item_first = 0;
    bool solo = false;                  // the current item (PVs never cross an item)
    bool ok = true;
    // PV of step s (both units) from V stage s % kPairVStages, issued by the elected lane; the
    // caller has waited for P(s), V(s) and, on an item's first PV, for the epilogue to have read
    // the previous item's O.
    auto pv_mmas = [&](uint32_t s, bool first) {
      const uint32_t sbuf = s % 3;
      const int vs = kPairKStages + (int)(s % kPairVStages);
      {
        const uint64_t va = kdesc0 + (uint64_t)((vs * kStageBytes) >> 4);
        const uint64_t vb = va + (uint64_t)(kKBytes >> 4);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          mma_bf16_ts(tcol + 192, tcol + 64 * sbuf + 8 * kk, va + (uint64_t)((2048 * kk) >> 4), kIdescPV64,
                      (first && kk == 0) ? 0u : 1u);
        if (!solo) {
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            mma_bf16_ts(tcol + 192 + kLane16, tcol + 64 * sbuf + 8 * kk + kLane16,
                        vb + (uint64_t)((2048 * kk) >> 4), kIdescPV64, (first && kk == 0) ? 0u : 1u);
        }
        mma_commit(&bars->o_done[X][s & 1]);
        mma_commit(&bars->kv_empty[X][vs]);
      }
    };
    auto issue_pv = [&]() -> bool {
      const uint32_t s = pvs;
      if (!warp_mbar_wait2(&bars->p_full[X][s % 3], (s / 3) & 1, &bars->kv_full[X][kPairKStages + s % kPairVStages],
                           (s / kPairVStages) & 1, true, abort))
        return false;
      const bool first = (s == item_first);
      if (first && titems > 0 && !warp_mbar_wait(&bars->o_free[X], (titems - 1) & 1, abort)) return false;
      tc_fence_after();
      if (elect_one()) pv_mmas(s, first);
      __syncwarp();
      ++pvs;
      return true;
    };
    // Taking an item reads its work entry and counts its steps (the MMAs need nothing else of
    // the entry list: K and V stages follow the step index).  The next item is taken while this
    // item's last PVs wait for their P, when the scheduler has already published it, so its
    // first QK follows the last PV directly.
    struct Taken {
      int item, cnt;
      PItem w;
    };
    auto take = [&](uint32_t kk, Taken& t) -> bool {
      const int slot = kk & 1;
      if (!warp_mbar_wait(&bars->item_full[X][slot], (kk >> 1) & 1, abort)) return false;
      t.item = item_slot[slot];
      __syncwarp();
      if (elect_one()) mbar_arrive(&bars->item_empty[X][slot]);
      __syncwarp();
      t.cnt = 0;
      if (t.item >= 0) {
        t.w = decode_pair(a, t.item);
        int last = -1;
        t.cnt = count_steps(entries, t.w.e0, t.w.n, (t.w.j & 1) ? kFlagActive1 : kFlagActive0, last);
      }
      return true;
    };
    Taken cur, nxt;
    bool have_next = false;
    for (uint32_t k = 0; ok; ++k) {
      if (have_next) {
        cur = nxt;
        have_next = false;
      } else if (!take(k, cur)) {
        ok = false;
        break;
      }
      if (cur.item < 0) break;
      if (cur.cnt == 0) continue;
      const PItem& w = cur.w;
      const int qs = qk % kQSlots;
      if (!warp_mbar_wait(&bars->q_full[X][qs], (qk / kQSlots) & 1, abort)) { ok = false; break; }
      ++qk;
      const uint32_t qaddr = smem_u32(smem + kOffQ + (kQSlots * X + qs) * kQBytes);
      const uint64_t qda = sw128_desc(qaddr, 16, 1024), qdb = sw128_desc(qaddr + kQBytes / 2, 16, 1024);
      item_first = steps;
      solo = w.solo;
      // The MMAs need only the step count: K and V stages follow the step index.
      for (int t = 0; t < cur.cnt && ok; ++t) {
        const int ks = steps % kPairKStages;
        while (ok && pvs + kPairPvLag < steps) ok = issue_pv();
        if (!ok) break;
        const bool pv_now = pvs + kPairPvLag == steps;
        const uint32_t ps = pvs;
        const bool pv_first = pv_now && ps == item_first;
        if (pv_first && titems > 0 && !warp_mbar_wait(&bars->o_free[X], (titems - 1) & 1, abort)) { ok = false; break; }
        if (!warp_mbar_wait3(&bars->kv_full[X][ks], (steps / kPairKStages) & 1, &bars->p_full[X][ps % 3],
                             (ps / 3) & 1, &bars->kv_full[X][kPairKStages + ps % kPairVStages],
                             (ps / kPairVStages) & 1, pv_now, abort)) { ok = false; break; }
        const uint32_t sb = steps % 3;
        tc_fence_after();
        if (elect_one()) {
          if (pv_now) pv_mmas(ps, pv_first);
          const uint64_t ka = kdesc0 + (uint64_t)((ks * kStageBytes) >> 4);
          const uint64_t kb = ka + (uint64_t)(kKBytes >> 4);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            mma_bf16_ss(tcol + 64 * sb, qda + 2 * kk, ka + 2 * kk, kIdescQK64, kk > 0 ? 1u : 0u);
          if (!solo) {
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              mma_bf16_ss(tcol + 64 * sb + kLane16, qdb + 2 * kk, kb + 2 * kk, kIdescQK64, kk > 0 ? 1u : 0u);
          }
          mma_commit(&bars->s_full[X][sb]);
          mma_commit(&bars->kv_empty[X][ks]);
          if (t == cur.cnt - 1) mma_commit(&bars->q_empty[X][qs]);
        }
        __syncwarp();
        if (pv_now) ++pvs;
        ++steps;
      }
      if (!ok) break;
      if (__all_sync(0xffffffffu, mbar_test_wait(&bars->item_full[X][(k + 1) & 1], ((k + 1) >> 1) & 1))) {
        if (!take(k + 1, nxt)) { ok = false; break; }
        have_next = true;
      }
      while (ok && pvs < steps) ok = issue_pv();
      if (!ok) break;
      if (steps > item_first) ++titems;
    }
    if (!ok && lane == 0) fail(abort, 3);
    if (elect_one()) mma_commit(&bars->drain);
    __syncwarp();
    if (lane == 0) {
      const uint64_t t0 = global_timer_ns();
      while (!mbar_try_wait(&bars->drain, 0) && global_timer_ns() - t0 < kWaitLimitNs) {
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------------ softmax + epilogue
    const int X = warp >> 2;                 // tile worker
    const bool upper = lane >= 16;           // partner unit's lanes
    const int r64 = 16 * (warp & 3) + (lane & 15);   // query row within chunk j
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    const uint32_t tcol = tmem + 256 * X;
    volatile int* item_slot = item_slots + 2 * X;
    uint64_t* s_full = bars->s_full[X];
    uint64_t* p_full = bars->p_full[X];
    uint64_t* o_done = bars->o_done[X];
    uint64_t* o_free = &bars->o_free[X];
    uint32_t it = 0, sb_c = 0, ph_c = 0;
    bool s_ready = false;
    uint32_t ep_phase = 0;                 // uses of ep_bar[X]
    bool ok = true;
    // The next item's id, work entry and first 32 entries are read before this item's epilogue
    // when the scheduler has already published it (the reads overlap the wait for the last PV).
    int n_item = -1;
    int32_t n_wk = 0, n_eb = 0;
    bool have_next = false;
    auto entries0 = [&](int32_t wkx) {
      const int e0 = work_word(wkx, 3), n = work_word(wkx, 4) - e0;
      return lane < n ? entries[e0 + lane] : 0;
    };
    for (uint32_t k = 0; ok; ++k) {
      int item;
      int32_t wk, eb0;
      if (have_next) {
        item = n_item;
        wk = n_wk;
        eb0 = n_eb;
        have_next = false;
      } else {
        const int slot = k & 1;
        if (!warp_mbar_wait(&bars->item_full[X][slot], (k >> 1) & 1, abort)) { ok = false; break; }
        item = item_slot[slot];
        mbar_arrive(&bars->item_empty[X][slot]);
        if (item < 0) break;
        wk = work_lanes(a, item);
        eb0 = entries0(wk);
      }
      if (item < 0) break;
      const int we0 = work_word(wk, 3), wn = work_word(wk, 4) - we0, wj = work_word(wk, 2);
      const int32_t fa = (wj & 1) ? kFlagActive1 : kFlagActive0;
      const int32_t fd = (wj & 1) ? kFlagDiag1 : kFlagDiag0;
      const bool live = !(work_word(wk, 1) < 0 && upper);
      float m = -INFINITY, l = 0.f;
      int nsteps = 0;
      for (int b0 = 0; b0 < wn && ok; b0 += 32) {
        const int32_t eb = b0 == 0 ? eb0 : (b0 + lane < wn ? entries[we0 + b0 + lane] : 0);
        uint32_t own = __ballot_sync(0xffffffffu, (eb & fa) != 0);
        while (own) {
          const int32_t e = __shfl_sync(0xffffffffu, eb, __ffs(own) - 1);
          own &= own - 1;
          ++nsteps;
          const uint32_t sb = sb_c;
          if (!s_ready && !warp_mbar_wait(&s_full[sb], ph_c, abort)) { ok = false; break; }
          tc_fence_after();
          uint32_t sr[64];
          XSAKE_TMEM_LD32(tcol + lane_base + 64 * sb, sr);
          XSAKE_TMEM_LD32(tcol + lane_base + 64 * sb + 32, (sr + 32));
          const bool next_done = mbar_test_wait(&s_full[sb_c == 2 ? 0 : sb_c + 1], sb_c == 2 ? ph_c ^ 1u : ph_c);
          XSAKE_TMEM_WAIT_LD32(sr);
          XSAKE_TMEM_WAIT_LD32((sr + 32));
          s_ready = __all_sync(0xffffffffu, next_done);
          uint32_t pk[32];
          float* x = reinterpret_cast<float*>(sr);   // raw scores
          // Keys past the token-level causal cut on the diagonal chunk, and every key of a
          // lane whose unit is absent (a lone unit), are masked.
          const int lim = !live ? -1 : ((e & fd) ? r64 : 63);
          if (__any_sync(0xffffffffu, lim < 63)) {
#pragma unroll
            for (int j = 0; j < 64; ++j)
              if (j > lim) x[j] = -INFINITY;
          }
          const float mx = rowmax64(x) * p.scale_log2;
          const bool need = (m != -INFINITY) && (mx > m + kRescaleThreshold);
          if (m == -INFINITY) m = mx;
          if (__any_sync(0xffffffffu, need)) {
            if (!warp_mbar_wait(&o_done[(it - 1) & 1], ((it - 1) >> 1) & 1, abort)) { ok = false; break; }
            tc_fence_after();
            const float alpha = need ? ex2(m - mx) : 1.0f;
            uint32_t orow[32];
#pragma unroll
            for (int hcol = 0; hcol < 2; ++hcol) {
              XSAKE_TMEM_LD32(tcol + lane_base + 192 + 32 * hcol, orow);
              XSAKE_TMEM_WAIT_LD32(orow);
#pragma unroll
              for (int j = 0; j < 32; ++j) orow[j] = __float_as_uint(__uint_as_float(orow[j]) * alpha);
              XSAKE_TMEM_ST32(tcol + lane_base + 192 + 32 * hcol, orow);
            }
            tmem_wait_st();
            if (need) {
              l *= alpha;
              m = mx;
            }
          }
          const float msub = (m == -INFINITY) ? 0.f : m;
          const uint64_t cc = pk2(p.scale_log2, p.scale_log2), nm = pk2(-msub, -msub);
          uint64_t acc[4] = {0ull, 0ull, 0ull, 0ull};
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            float x0, x1, p0, p1;
            upk2(fma2(pk2(x[2 * j], x[2 * j + 1]), cc, nm), x0, x1);
            if ((j & 7) < 2) {
              exp2_poly2(x0, x1, p0, p1);
            } else {
              p0 = ex2(x0);
              p1 = ex2(x1);
            }
            acc[j & 3] = add2(acc[j & 3], pk2(p0, p1));
            __nv_bfloat162 pb = __floats2bfloat162_rn(p0, p1);
            pk[j] = *reinterpret_cast<uint32_t*>(&pb);
            // The first 16 columns of P go out while the second half is computed, so only the
            // second store's latency is left before the arrive (A/B: ~1%, identical outputs).
            if (j == 15) XSAKE_TMEM_ST16(tcol + lane_base + 64 * sb, pk);
          }
          float s0, s1;
          upk2(add2(add2(acc[0], acc[1]), add2(acc[2], acc[3])), s0, s1);
          l += s0 + s1;
          XSAKE_TMEM_ST16(tcol + lane_base + 64 * sb + 16, (pk + 16));
          tmem_wait_st();
          tc_fence_before();
          mbar_arrive(&p_full[sb]);
          ++it;
          if (++sb_c == 3) {
            sb_c = 0;
            ph_c ^= 1;
          }
        }
      }
      if (!ok) break;
      if (__all_sync(0xffffffffu, mbar_test_wait(&bars->item_full[X][(k + 1) & 1], ((k + 1) >> 1) & 1))) {
        n_item = item_slot[(k + 1) & 1];
        mbar_arrive(&bars->item_empty[X][(k + 1) & 1]);
        if (n_item >= 0) {
          n_wk = work_lanes(a, n_item);
          n_eb = entries0(n_wk);
        }
        have_next = true;
      }
      // ---------------------------------------------------------------- epilogue
      float o[64];
      if (nsteps > 0) {
        // The same two-phase wait for the last PVs as in tile_roles.
        if (it >= 2 && !warp_mbar_wait(&o_done[(it - 2) & 1], ((it - 2) >> 1) & 1, abort)) { ok = false; break; }
        if (!warp_mbar_wait(&o_done[(it - 1) & 1], ((it - 1) >> 1) & 1, abort)) { ok = false; break; }
        tc_fence_after();
        load_o_row(tcol + lane_base + 192, o);
        tc_fence_before();
        mbar_arrive(o_free);
      } else {
#pragma unroll
        for (int j = 0; j < 64; ++j) o[j] = 0.f;
      }
      const int grp = work_word(wk, 6), parts = work_word(wk, 5);
      if (grp >= 0 && !split_finish(p, grp, parts >> 8, parts & 0xff, work_word(wk, 7), threadIdx.x & 127,
                                    &bars->ep_bar[X], ep_phase, c.ep_flag + X, m, l, o, abort, ok)) {
        if (!ok) break;
        continue;   // another piece of this item merges the rows
      }
      const int u0 = work_word(wk, 0), u1r = work_word(wk, 1), u1 = u1r < 0 ? u0 : u1r;
      PItem we;
      we.b0 = u0 / a.H; we.h0 = u0 % a.H; we.b1 = u1 / a.H; we.h1 = u1 % a.H; we.j = wj;
      const int bb = upper ? we.b1 : we.b0, hh = upper ? we.h1 : we.h0;
      const int tok = 64 * we.j + r64;
      const bool valid = live && tok < a.S;
      const bool empty = valid && !(l > 0.f);
      uint4* orow_g = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(a.o) + bb * a.os[0] +
                                               hh * a.os[1] + (int64_t)(valid ? tok : 0) * a.os[2]);
      if (valid && !empty) store_o_row(orow_g, o, 1.f / l, p.o_rows_32b);
      const bool empty_lo = __any_sync(0xffffffffu, empty && !upper);
      const bool empty_hi = __any_sync(0xffffffffu, empty && upper);
      if (empty_lo || empty_hi) {
        // Rows with no live score attend uniformly (the reference's finfo.min fill).
        float2 mean0 = make_float2(0.f, 0.f), mean1 = make_float2(0.f, 0.f);
        if (empty_lo) warp_mean_v(a, we.b0, we.h0, mean0);
        if (empty_hi) warp_mean_v(a, we.b1, we.h1, mean1);
#pragma unroll
        for (int cc = 0; cc < 8; ++cc) {
          uint32_t wv[4];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int src = 4 * cc + q;
            const float x0 = __shfl_sync(0xffffffffu, mean0.x, src), y0 = __shfl_sync(0xffffffffu, mean0.y, src);
            const float x1 = __shfl_sync(0xffffffffu, mean1.x, src), y1 = __shfl_sync(0xffffffffu, mean1.y, src);
            __nv_bfloat162 pb = __floats2bfloat162_rn(upper ? x1 : x0, upper ? y1 : y0);
            wv[q] = *reinterpret_cast<uint32_t*>(&pb);
          }
          if (empty) orow_g[cc] = make_uint4(wv[0], wv[1], wv[2], wv[3]);
        }
      }
      if (valid) a.lse[(int64_t)(bb * a.H + hh) * a.S + tok] = empty ? kMaskFill : (m + __log2f(l)) * kLn2;
    }
    if (!ok) fail(abort, 4);
  }
}

__global__ void __launch_bounds__(kThreads, 1)
tc_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
              const __grid_constant__ CUtensorMap tmV, const TcParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Bars* bars = reinterpret_cast<Bars*>(smem + kOffBar);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffMisc);
  volatile int* abort = reinterpret_cast<volatile int*>(smem + kOffMisc + 4);
  volatile int* plan_ok = reinterpret_cast<volatile int*>(smem + kOffMisc + 8);
  volatile int* item_slots = reinterpret_cast<volatile int*>(smem + kOffMisc + 16);   // [tile][slot]
  volatile int* ep_flag = reinterpret_cast<volatile int*>(smem + kOffMisc + 48);      // [tile]
  const AttnArgs& a = p.a;
  const PlanLayout& L = a.L;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    *abort = 0;
    *plan_ok = plan_matches(a) && a.plan[H_HAS_CSR] == 1;
    if (!*plan_ok) record_device_error(DEV_ERR_PLAN, 10);
    for (int s = 0; s < 2; ++s) {
      for (int t = 0; t < 2; ++t) {
        mbar_init(&bars->item_full[t][s], 1);
        mbar_init(&bars->item_empty[t][s], kItemReaders);
        mbar_init(&bars->q_full[t][s], 1);
        mbar_init(&bars->q_empty[t][s], 1);
      }
      mbar_init(&bars->o_free[s], 128);
      mbar_init(&bars->ep_bar[s], 128);
      for (int b = 0; b < 2; ++b) mbar_init(&bars->o_done[s][b], 1);
      for (int b = 0; b < 3; ++b) mbar_init(&bars->p_full[s][b], 128);
      for (int b = 0; b < 3; ++b) mbar_init(&bars->s_full[s][b], 1);
    }
    for (int t = 0; t < 2; ++t)
      for (int s = 0; s < kStages; ++s) {
        mbar_init(&bars->kv_full[t][s], 1);
        mbar_init(&bars->kv_empty[t][s], 1);
      }
    mbar_init(&bars->drain, 2);
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == 8 && lane == 0) {
    tma_prefetch_desc(&tmQ);
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

  if (*plan_ok) {
    const FwdCtx c{smem, bars, abort, item_slots, ep_flag, tmem, a.plan + L.f_entries_off};
    // The plan compiler chose the pairing from the mask (H_FWD_PAIR); every CTA reads the same word.
    if (a.plan[H_FWD_PAIR] == kPairUnits)
      pair_roles(tmQ, tmK, tmV, p, c);
    else
      tile_roles(tmQ, tmK, tmV, p, c);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

constexpr int kMaxDev = 64;
std::once_flag g_attr_once[kMaxDev];
cudaError_t g_attr_err[kMaxDev];

}  // namespace

// ------------------------------------------------------------------------------ host side
namespace {
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

int get_encoder(PFN_cuTensorMapEncodeTiled_v12000* fn) {
  cudaError_t err = cudaSuccess;
  std::call_once(g_encode_once, [&] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    err = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q);
    if (err == cudaSuccess && q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  XSAKE_REQUIRE(g_encode != nullptr, XSAKE_ECUDA, "cuTensorMapEncodeTiled unavailable (%s)",
                cudaGetErrorString(err));
  *fn = g_encode;
  return XSAKE_OK;
}

}  // namespace

// 4-D bf16 map over [B, H, S, 64] with arbitrary (b, h, s) strides; box = `rows` x 64.
// Dimensions are ordered by increasing stride, as the tiled TMA layout expects.
int tc_make_map(CUtensorMap* map, const void* base, const int64_t st[3], int B, int H, int S, int rows) {
  PFN_cuTensorMapEncodeTiled_v12000 enc;
  int s = get_encoder(&enc);
  if (s) return s;
  // Dimensions (d, s, h, b) in the kernels' coordinate order with the caller's strides, whatever
  // their order: [B, H, S, D] and the projection layout [B, S, H, D] both load as 64-column
  // tiles of `rows` consecutive tokens.
  cuuint64_t dims[4] = {64, (cuuint64_t)S, (cuuint64_t)H, (cuuint64_t)B};
  cuuint64_t strides[3] = {(cuuint64_t)st[2] * 2, (cuuint64_t)st[1] * 2, (cuuint64_t)st[0] * 2};
  cuuint32_t box[4] = {64, (cuuint32_t)rows, 1, 1};
  cuuint32_t es[4] = {1, 1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box, es,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  XSAKE_REQUIRE(r == CUDA_SUCCESS, XSAKE_ECUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return XSAKE_OK;
}

bool tc_attn_fwd_supported(const AttnArgs& a, int dtype) {
  if (dtype != XSAKE_BF16 || a.D != 64 || !a.L.has_csr) return false;
  auto aligned = [](const void* ptr, const int64_t* st) {
    return ((uintptr_t)ptr & 15) == 0 && st[0] % 8 == 0 && st[1] % 8 == 0 && st[2] % 8 == 0;
  };
  if (!(aligned(a.q, a.qs) && aligned(a.k, a.ks) && aligned(a.v, a.vs) && aligned(a.o, a.os))) return false;
  // Layouts the TMA unit accepts are taken; anything it rejects goes to the CUDA-core kernels.
  CUtensorMap m;
  const bool ok = tc_make_map(&m, a.q, a.qs, a.B, a.H, a.S, 128) == XSAKE_OK &&
                  tc_make_map(&m, a.k, a.ks, a.B, a.H, a.S, 128) == XSAKE_OK &&
                  tc_make_map(&m, a.v, a.vs, a.B, a.H, a.S, 128) == XSAKE_OK;
  clear_error();
  return ok;
}

// Workspace: work-item counter (256 B) | split-group counters (kSplitSlots ints, reset with the
// counter) | kSplitSlots partial slots of kSlotFloats floats.
constexpr size_t kFwdGroupOff = 256;
constexpr size_t kFwdResetBytes = kFwdGroupOff + 4 * kSplitSlots;
constexpr size_t kFwdPartOff = (kFwdResetBytes + 255) / 256 * 256;
constexpr size_t kFwdWsBytes = kFwdPartOff + (size_t)kSplitSlots * kSlotFloats * 4;

size_t tc_attn_fwd_workspace() { return kFwdWsBytes; }

int tc_attn_fwd(const AttnArgs& a, void* ws, size_t ws_bytes, cudaStream_t s) {
  DeviceInfo di;
  int st = device_info(&di);
  if (st) return st;
  XSAKE_REQUIRE(di.major == 10, XSAKE_EUNSUPPORTED, "tensor-core path needs sm_100 (got sm_%d%d)", di.major,
                di.minor);
  XSAKE_REQUIRE(ws != nullptr && ws_bytes >= kFwdWsBytes && ((uintptr_t)ws & 255) == 0, XSAKE_EINVAL,
                "the tensor-core forward needs a %zu-byte, 256-byte aligned workspace (got %zu bytes)", kFwdWsBytes,
                ws_bytes);
  // The plan (H_FWD_PAIR) chooses the pairing on the device; the grid covers either item count.
  CUtensorMap mq, mk, mv;
  if ((st = tc_make_map(&mq, a.q, a.qs, a.B, a.H, a.S, 64))) return st;
  if ((st = tc_make_map(&mk, a.k, a.ks, a.B, a.H, a.S, 64))) return st;
  if ((st = tc_make_map(&mv, a.v, a.vs, a.B, a.H, a.S, 64))) return st;
  int dev = 0;
  XSAKE_CUDA_TRY(cudaGetDevice(&dev));
  XSAKE_REQUIRE(dev < kMaxDev, XSAKE_EUNSUPPORTED, "device ordinal %d", dev);
  std::call_once(g_attr_once[dev], [dev] {
    g_attr_err[dev] = cudaFuncSetAttribute(tc_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
  });
  XSAKE_REQUIRE(g_attr_err[dev] == cudaSuccess, XSAKE_ECUDA, "cudaFuncSetAttribute: %s",
                cudaGetErrorString(g_attr_err[dev]));
  TcParams p;
  p.a = a;
  p.scale_log2 = a.scale * kLog2e;
  p.o_rows_32b = ((uintptr_t)a.o & 31) == 0 && a.os[0] % 16 == 0 && a.os[1] % 16 == 0 && a.os[2] % 16 == 0;
  p.counter = reinterpret_cast<int*>(ws);
  p.grp_counter = reinterpret_cast<int*>(reinterpret_cast<uint8_t*>(ws) + kFwdGroupOff);
  p.parts = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(ws) + kFwdPartOff);
  XSAKE_CUDA_TRY(cudaMemsetAsync(ws, 0, kFwdResetBytes, s));
  // Work items: at most the plan's table size (the count itself is on the device).
  const int grid = std::max(1, std::min((a.L.max_work + 1) / 2, di.sm_count));
  tc_fwd_kernel<<<grid, kThreads, kSmemBytes, s>>>(mq, mk, mv, p);
  return check_launch("tc_fwd_kernel");
}

}  // namespace xsake
