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
// Work item = 128 query rows (two 64-row chunks 2t, 2t+1 of one (b, h)) and the union of their
// active 64-key chunks.  Per chunk: S = Q K^T (tcgen05, M=128 N=64 K=64, fp32 in TMEM),
// softmax by one thread per row straight out of TMEM, P (bf16) to shared memory, O += P V
// (tcgen05, fp32 accumulator resident in TMEM).  Roles per CTA (192 threads):
//   warps 0-3  softmax + epilogue, thread i owns row i (TMEM lane i)
//   warp 4     TMA producer: Q tile once per item, K/V chunks into a 4-stage ring
//   warp 5     MMA issuer (one thread): QK of chunk i+1 is queued before PV of chunk i
// Two CTAs per SM (97 KB smem, 256 TMEM columns each) so one CTA's softmax overlaps the
// other's MMAs.  The running max is only moved when it grows by more than 2^8 (rescaling O in
// TMEM is then rare); exp2 runs on the MUFU unit.  Items are taken in descending-cost order
// with a boustrophedon assignment over the persistent CTAs.
#include "attn_common.cuh"
#include "sm100.cuh"

#include <cudaTypedefs.h>
#include <algorithm>
#include <mutex>

XSAKE_DEFINE_DEVICE_ERROR(tcfwd)

namespace xsake {
namespace {

using namespace sm100;

constexpr int kStages = 4;
constexpr int kThreads = 192;
constexpr int kQBytes = 128 * 64 * 2;
constexpr int kKBytes = 64 * 64 * 2;
constexpr int kStageBytes = 2 * kKBytes;
constexpr int kOffQ = 0;
constexpr int kOffKV = kOffQ + kQBytes;
constexpr int kOffP = kOffKV + kStages * kStageBytes;
constexpr int kOffBar = kOffP + kQBytes;
constexpr int kNumBars = 2 + 2 * kStages + 2 + 2 + 4;
constexpr int kOffMisc = kOffBar + kNumBars * 8;
constexpr int kSmemBytes = kOffMisc + 64 + 1024;  // + alignment slack
constexpr uint32_t kTmemCols = 256;               // S0 [0,64) S1 [64,128) O [128,192)
constexpr uint32_t kIdescQK = idesc_bf16(128, 64, false);
constexpr uint32_t kIdescPV = idesc_bf16(128, 64, true);
constexpr float kRescaleThreshold = 8.0f;          // log2 units

struct Bars {
  uint64_t q_full, q_empty;
  uint64_t kv_full[kStages], kv_empty[kStages];
  uint64_t s_full[2], s_free[2];
  uint64_t p_full, o_done, o_free, drain;
};
static_assert(sizeof(Bars) == kNumBars * 8, "barrier block size");

struct TcParams {
  AttnArgs a;
  float scale_log2;
};

__device__ __forceinline__ int snake_rank(int round, int cta, int G) {
  return round * G + ((round & 1) ? (G - 1 - cta) : cta);
}

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

__global__ void __launch_bounds__(kThreads, 2)
tc_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
              const __grid_constant__ CUtensorMap tmV, const TcParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Bars* bars = reinterpret_cast<Bars*>(smem + kOffBar);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffMisc);
  volatile int* abort = reinterpret_cast<volatile int*>(smem + kOffMisc + 4);
  volatile int* plan_ok = reinterpret_cast<volatile int*>(smem + kOffMisc + 8);
  const AttnArgs& a = p.a;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    *abort = 0;
    *plan_ok = plan_matches(a) && a.plan[H_HAS_CSR] == 1;
    if (!*plan_ok) record_device_error(DEV_ERR_PLAN, 10);
    mbar_init(&bars->q_full, 1);
    mbar_init(&bars->q_empty, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars->kv_full[s], 1);
      mbar_init(&bars->kv_empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bars->s_full[s], 1);
      mbar_init(&bars->s_free[s], 128);
    }
    mbar_init(&bars->p_full, 128);
    mbar_init(&bars->o_done, 1);
    mbar_init(&bars->o_free, 128);
    mbar_init(&bars->drain, 1);
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == 4 && lane == 0) {
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

  const PlanLayout& L = a.L;
  const int32_t* rowptr = a.plan + L.f_rowptr_off;
  const int32_t* entries = a.plan + L.f_entries_off;
  const int32_t* items = a.plan + L.f_items_off;
  const int G = gridDim.x, cta = blockIdx.x;

  if (*plan_ok) {
    if (warp == 4) {
      // ------------------------------------------------------------------ TMA producer
      if (lane == 0) {
        uint32_t it = 0, jj = 0;
        for (int round = 0;; ++round) {
          const int rank = snake_rank(round, cta, G);
          if (rank >= L.nitems || *abort) break;
          const int item = items[rank];
          const int t = item % L.npairs, bh = item / L.npairs, b = bh / a.H, h = bh % a.H;
          const int r = L.group_of(b, h) * L.npairs + t;
          const int e0 = rowptr[r], n = rowptr[r + 1] - e0;
          if (n == 0) continue;
          if (!mbar_wait(&bars->q_empty, (jj & 1) ^ 1, abort)) { fail(abort, 1); break; }
          mbar_arrive_expect_tx(&bars->q_full, kQBytes);
          tma_load_4d(smem + kOffQ, &tmQ, &bars->q_full, 0, 128 * t, h, b);
          bool ok = true;
          for (int i = 0; i < n; ++i, ++it) {
            const int st = it % kStages;
            if (!mbar_wait(&bars->kv_empty[st], ((it / kStages) & 1) ^ 1, abort)) { ok = false; break; }
            const int c = entries[e0 + i] & kEntryIdxMask;
            uint8_t* kbuf = smem + kOffKV + st * kStageBytes;
            mbar_arrive_expect_tx(&bars->kv_full[st], kStageBytes);
            tma_load_4d(kbuf, &tmK, &bars->kv_full[st], 0, 64 * c, h, b);
            tma_load_4d(kbuf + kKBytes, &tmV, &bars->kv_full[st], 0, 64 * c, h, b);
          }
          if (!ok) { fail(abort, 2); break; }
          ++jj;
        }
        // Every load issued above has been consumed by the MMA warp on the normal path; on
        // the abort path give in-flight copies a bounded chance to land before exit.
        if (*abort) {
          for (int s = 0; s < kStages; ++s) {
            const uint64_t t0 = global_timer_ns();
            while (!mbar_try_wait(&bars->kv_full[s], 0) && !mbar_try_wait(&bars->kv_full[s], 1) &&
                   global_timer_ns() - t0 < 1000000ull) {
            }
          }
        }
      }
    } else if (warp == 5) {
      // ------------------------------------------------------------------ MMA issuer
      if (lane == 0) {
        const uint32_t q_addr = smem_u32(smem + kOffQ);
        const uint32_t p_addr = smem_u32(smem + kOffP);
        const uint64_t qdesc = sw128_desc(q_addr, 16, 1024);
        const uint64_t pdesc = sw128_desc(p_addr, 16, 1024);
        uint32_t it = 0, jj = 0;
        bool ok = true;
        auto issue_pv = [&](uint32_t x, bool first) -> bool {
          if (!mbar_wait(&bars->p_full, x & 1, abort)) return false;
          if (first && jj > 0 && !mbar_wait(&bars->o_free, (jj - 1) & 1, abort)) return false;
          tc_fence_after();
          const int st = x % kStages;
          const uint32_t v_addr = smem_u32(smem + kOffKV + st * kStageBytes + kKBytes);
          const uint64_t vdesc = sw128_desc(v_addr, 16, 1024);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            mma_bf16_ss(tmem + 128, pdesc + 2 * kk, vdesc + (uint64_t)((2048 * kk) >> 4), kIdescPV,
                        (first && kk == 0) ? 0u : 1u);
          mma_commit(&bars->o_done);
          mma_commit(&bars->kv_empty[st]);
          return true;
        };
        for (int round = 0; ok; ++round) {
          const int rank = snake_rank(round, cta, G);
          if (rank >= L.nitems || *abort) break;
          const int item = items[rank];
          const int t = item % L.npairs, bh = item / L.npairs;
          const int r = L.group_of(bh / a.H, bh % a.H) * L.npairs + t;
          const int n = rowptr[r + 1] - rowptr[r];
          if (n == 0) continue;
          if (!mbar_wait(&bars->q_full, jj & 1, abort)) { ok = false; break; }
          for (int i = 0; i < n && ok; ++i, ++it) {
            const int st = it % kStages;
            const uint32_t sb = it & 1;
            if (!mbar_wait(&bars->kv_full[st], (it / kStages) & 1, abort) ||
                !mbar_wait(&bars->s_free[sb], ((it >> 1) & 1) ^ 1, abort)) { ok = false; break; }
            tc_fence_after();
            const uint64_t kdesc = sw128_desc(smem_u32(smem + kOffKV + st * kStageBytes), 16, 1024);
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              mma_bf16_ss(tmem + 64 * sb, qdesc + 2 * kk, kdesc + 2 * kk, kIdescQK, kk > 0 ? 1u : 0u);
            mma_commit(&bars->s_full[sb]);
            if (i == n - 1) mma_commit(&bars->q_empty);
            if (i > 0 && !issue_pv(it - 1, i == 1)) { ok = false; break; }
          }
          if (!ok) break;
          if (!issue_pv(it - 1, n == 1)) { ok = false; break; }
          ++jj;
        }
        if (!ok) fail(abort, 3);
        // Drain: no MMA may be in flight when TMEM is released.
        mma_commit(&bars->drain);
        const uint64_t t0 = global_timer_ns();
        while (!mbar_try_wait(&bars->drain, 0) && global_timer_ns() - t0 < kWaitLimitNs) {
        }
      }
    } else {
      // ------------------------------------------------------------------ softmax + epilogue
      const int row = threadIdx.x;          // 0..127, TMEM lane
      const int half = row >> 6;
      const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
      const int32_t f_active = half ? kFlagActive1 : kFlagActive0;
      const int32_t f_diag = half ? kFlagDiag1 : kFlagDiag0;
      const int diag_lim = row & 63;
      uint8_t* prow = smem + kOffP + (row >> 3) * 1024 + (row & 7) * 128;
      const int rsw = row & 7;
      uint32_t it = 0, jj = 0;
      bool ok = true;
      for (int round = 0; ok; ++round) {
        const int rank = snake_rank(round, cta, G);
        if (rank >= L.nitems || *abort) break;
        const int item = items[rank];
        const int t = item % L.npairs, bh = item / L.npairs, b = bh / a.H, h = bh % a.H;
        const int r = L.group_of(b, h) * L.npairs + t;
        const int e0 = rowptr[r], n = rowptr[r + 1] - e0;
        float m = -INFINITY, l = 0.f;
        int32_t e_next = n > 0 ? entries[e0] : 0;
        for (int i = 0; i < n; ++i, ++it) {
          const int32_t e = e_next;
          if (i + 1 < n) e_next = entries[e0 + i + 1];   // prefetch: off the critical path
          const uint32_t sb = it & 1;
          if (!warp_mbar_wait(&bars->s_full[sb], (it >> 1) & 1, abort)) { ok = false; break; }
          tc_fence_after();
          uint32_t sr[64];
          XSAKE_TMEM_LD32(tmem + lane_base + 64 * sb, sr);
          XSAKE_TMEM_LD32(tmem + lane_base + 64 * sb + 32, (sr + 32));
          XSAKE_TMEM_WAIT_LD32(sr);
          XSAKE_TMEM_WAIT_LD32((sr + 32));
          tc_fence_before();
          mbar_arrive(&bars->s_free[sb]);
          bool waited = false;
          uint32_t pk[32];
          if (e & f_active) {
            float* x = reinterpret_cast<float*>(sr);   // raw scores
            if (e & f_diag) {                          // warp-uniform: token-level causal cut
#pragma unroll
              for (int j = 0; j < 64; ++j)
                if (j > diag_lim) x[j] = -INFINITY;
            }
            // Row max of the raw scores: a depth-4 tree of 3-input maxes.
            float t1[22];
#pragma unroll
            for (int j = 0; j < 21; ++j) t1[j] = max3(x[3 * j], x[3 * j + 1], x[3 * j + 2]);
            t1[21] = x[63];
            float t2[8];
#pragma unroll
            for (int j = 0; j < 7; ++j) t2[j] = max3(t1[3 * j], t1[3 * j + 1], t1[3 * j + 2]);
            t2[7] = t1[21];
            const float mraw = fmaxf(max3(t2[0], t2[1], t2[2]), max3(t2[3], t2[4], fmaxf(t2[5], fmaxf(t2[6], t2[7]))));
            const float mx = mraw * p.scale_log2;       // log2 units (scale > 0)
            const bool need = (m != -INFINITY) && (mx > m + kRescaleThreshold);
            if (m == -INFINITY) m = mx;
            // TMEM loads/stores are warp-collective: the whole warp rescales when any row must.
            if (__any_sync(0xffffffffu, need)) {
              // O holds PV of earlier chunks: wait for the last one, then rescale in TMEM.
              if (!warp_mbar_wait(&bars->o_done, (it - 1) & 1, abort)) { ok = false; break; }
              waited = true;
              tc_fence_after();
              const float alpha = need ? ex2(m - mx) : 1.0f;
              uint32_t orow[32];
#pragma unroll
              for (int hcol = 0; hcol < 2; ++hcol) {
                XSAKE_TMEM_LD32(tmem + lane_base + 128 + 32 * hcol, orow);
                XSAKE_TMEM_WAIT_LD32(orow);
#pragma unroll
                for (int j = 0; j < 32; ++j) orow[j] = __float_as_uint(__uint_as_float(orow[j]) * alpha);
                XSAKE_TMEM_ST32(tmem + lane_base + 128 + 32 * hcol, orow);
              }
              tmem_wait_st();
              if (need) {
                l *= alpha;
                m = mx;
              }
            }
            const float msub = (m == -INFINITY) ? 0.f : m;   // no live score yet: every x is -inf
            // p = 2^(s*scale*log2e - m): one packed FMA per pair; 3 of every 8 pairs go through
            // the polynomial exp2 on the FMA/ALU pipes, the rest through MUFU ex2.
            const uint64_t cc = pk2(p.scale_log2, p.scale_log2), nm = pk2(-msub, -msub);
            uint64_t acc[4] = {0ull, 0ull, 0ull, 0ull};
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              float x0, x1, p0, p1;
              upk2(fma2(pk2(x[2 * j], x[2 * j + 1]), cc, nm), x0, x1);
              if ((j & 7) < 3) {
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
          // PV of the previous chunk reads the P buffer: wait for it before overwriting.
          if (it > 0 && !waited && !warp_mbar_wait(&bars->o_done, (it - 1) & 1, abort)) { ok = false; break; }
#pragma unroll
          for (int cc = 0; cc < 8; ++cc)
            *reinterpret_cast<uint4*>(prow + ((cc ^ rsw) << 4)) =
                make_uint4(pk[4 * cc], pk[4 * cc + 1], pk[4 * cc + 2], pk[4 * cc + 3]);
          fence_proxy_async_smem();
          tc_fence_before();
          mbar_arrive(&bars->p_full);
        }
        if (!ok) break;
        // ---------------------------------------------------------------- epilogue
        const int tok = 128 * t + row;
        const bool valid = tok < a.S;
        const bool empty = valid && !(l > 0.f);
        uint4* orow_g = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(a.o) + b * a.os[0] +
                                                 h * a.os[1] + (int64_t)(valid ? tok : 0) * a.os[2]);
        if (n > 0) {
          if (!warp_mbar_wait(&bars->o_done, (it - 1) & 1, abort)) { ok = false; break; }
          tc_fence_after();
          const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll
          for (int hcol = 0; hcol < 2; ++hcol) {
            uint32_t orow[32];
            XSAKE_TMEM_LD32(tmem + lane_base + 128 + 32 * hcol, orow);
            XSAKE_TMEM_WAIT_LD32(orow);
            if (valid && !empty) {
#pragma unroll
              for (int cc = 0; cc < 4; ++cc) {
                uint32_t w[4];
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                  __nv_bfloat162 pb = __floats2bfloat162_rn(__uint_as_float(orow[8 * cc + 2 * q]) * inv,
                                                            __uint_as_float(orow[8 * cc + 2 * q + 1]) * inv);
                  w[q] = *reinterpret_cast<uint32_t*>(&pb);
                }
                orow_g[4 * hcol + cc] = make_uint4(w[0], w[1], w[2], w[3]);
              }
            }
          }
          tc_fence_before();
          mbar_arrive(&bars->o_free);
          ++jj;
        }
        if (__any_sync(0xffffffffu, empty)) {
          // Rows with no live score: the reference's finfo.min fill makes them attend uniformly.
          float2 mine;
          warp_mean_v(a, b, h, mine);
#pragma unroll
          for (int cc = 0; cc < 8; ++cc) {
            uint32_t w[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const int src = 4 * cc + q;   // column pair index 0..31
              __nv_bfloat162 pb = __floats2bfloat162_rn(__shfl_sync(0xffffffffu, mine.x, src),
                                                        __shfl_sync(0xffffffffu, mine.y, src));
              w[q] = *reinterpret_cast<uint32_t*>(&pb);
            }
            if (empty) orow_g[cc] = make_uint4(w[0], w[1], w[2], w[3]);
          }
        }
        if (valid) a.lse[(int64_t)bh * a.S + tok] = empty ? kMaskFill : (m + __log2f(l)) * kLn2;
      }
      if (!ok) fail(abort, 4);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ------------------------------------------------------------------------------ host side
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

// 4-D bf16 map over [B, H, S, 64] with arbitrary (b, h, s) strides; box = `rows` x 64.
// Dimensions are ordered by increasing stride, as the tiled TMA layout expects.
int make_map(CUtensorMap* map, const void* base, const int64_t st[3], int B, int H, int S, int rows) {
  PFN_cuTensorMapEncodeTiled_v12000 enc;
  int s = get_encoder(&enc);
  if (s) return s;
  struct Dim { cuuint64_t size; cuuint64_t stride; cuuint32_t box; };
  Dim d[3] = {{(cuuint64_t)S, (cuuint64_t)st[2] * 2, (cuuint32_t)rows},
              {(cuuint64_t)H, (cuuint64_t)st[1] * 2, 1},
              {(cuuint64_t)B, (cuuint64_t)st[0] * 2, 1}};
  std::stable_sort(d, d + 3, [](const Dim& x, const Dim& y) { return x.stride < y.stride; });
  cuuint64_t dims[4] = {64, d[0].size, d[1].size, d[2].size};
  cuuint64_t strides[3] = {d[0].stride, d[1].stride, d[2].stride};
  cuuint32_t box[4] = {64, d[0].box, d[1].box, d[2].box};
  cuuint32_t es[4] = {1, 1, 1, 1};
  // The kernel addresses tiles as (d, s, h, b); only the canonical order is implemented.
  XSAKE_REQUIRE(d[0].box == (cuuint32_t)rows, XSAKE_EUNSUPPORTED,
                "the sequence stride must be the smallest of the (b, h, s) strides");
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box, es,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  XSAKE_REQUIRE(r == CUDA_SUCCESS, XSAKE_ECUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return XSAKE_OK;
}

}  // namespace

bool tc_attn_fwd_supported(const AttnArgs& a, int dtype) {
  if (dtype != XSAKE_BF16 || a.D != 64 || !a.L.has_csr) return false;
  auto aligned = [](const void* ptr, const int64_t* st) {
    return ((uintptr_t)ptr & 15) == 0 && st[0] % 8 == 0 && st[1] % 8 == 0 && st[2] % 8 == 0 &&
           st[2] > 0 && st[2] <= st[1] && st[2] <= st[0];
  };
  return aligned(a.q, a.qs) && aligned(a.k, a.ks) && aligned(a.v, a.vs) && aligned(a.o, a.os);
}

size_t tc_attn_fwd_workspace(const AttnArgs&) { return 0; }

int tc_attn_fwd(const AttnArgs& a, void*, size_t, cudaStream_t s) {
  DeviceInfo di;
  int st = device_info(&di);
  if (st) return st;
  XSAKE_REQUIRE(di.major == 10, XSAKE_EUNSUPPORTED, "tensor-core path needs sm_100 (got sm_%d%d)", di.major,
                di.minor);
  CUtensorMap mq, mk, mv;
  if ((st = make_map(&mq, a.q, a.qs, a.B, a.H, a.S, 128))) return st;
  if ((st = make_map(&mk, a.k, a.ks, a.B, a.H, a.S, 64))) return st;
  if ((st = make_map(&mv, a.v, a.vs, a.B, a.H, a.S, 64))) return st;
  static std::once_flag attr_once;
  cudaError_t aerr = cudaSuccess;
  std::call_once(attr_once, [&] {
    aerr = cudaFuncSetAttribute(tc_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
  });
  XSAKE_REQUIRE(aerr == cudaSuccess, XSAKE_ECUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(aerr));
  TcParams p;
  p.a = a;
  p.scale_log2 = a.scale * kLog2e;
  const int nitems = a.L.nitems;
  const int grid = std::max(1, std::min(nitems, 2 * di.sm_count));
  tc_fwd_kernel<<<grid, kThreads, kSmemBytes, s>>>(mq, mk, mv, p);
  return check_launch("tc_fwd_kernel");
}

}  // namespace xsake
