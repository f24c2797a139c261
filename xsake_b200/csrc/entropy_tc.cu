// Fused QK -> entropy on the sm_100a tensor cores: compute_attention_entropy
// (kernels/hads/hads_pattern.py:36-50) of softmax(Q K^T * scale) over all S keys, summed per head
// in fp64, without materialising P; or of the masked weights sparse_attention_reference returns
// (kernels/pallas/sparse_attention.py:76-87: block mask, causal cut, finfo.min fill), which the
// reference's calibration collects from layer 0 (training/trainer.py:79-117).  The entry points
// are xsake_entropy_qk and xsake_attn_entropy (attn_probs.cu), which run this kernel for
// head_dim 64 and keep the CUDA-core kernel for the other shapes.
//
// Precision.  Scores must be fp32-accurate (a TF32 product moves entropies by ~1e-3), so an fp32
// operand x is split into three bf16 parts x = x1 + x2 + x3 (x1 = bf16(x), x2 = bf16(x - x1),
// x3 = bf16(x - x1 - x2); each remainder is exact in fp32) and a score is the fp32 accumulation
// of the six bf16 products whose size is at least 2^-16 of the leading one:
// q3 k1 + q1 k3 + q2 k2 + q2 k1 + q1 k2 + q1 k1 (bf16 products are exact, so the error is that of
// the dropped terms, ~2^-24, plus the accumulation).  bf16 inputs need only q1 k1.
//
// Layout.  CTA = 128 query rows of one (b, h), 192 threads: warps 0-3 own one row each per thread
// (TMEM lane = row), warp 4 loads K chunks with TMA, warp 5 issues the MMAs.  The row threads
// write their row's Q parts into TMEM (A operand, 32 columns per part); K parts arrive per
// 64-key chunk in a 4-stage ring (3 x 8 KB a stage, SWIZZLE_128B).  S = Q K^T of a chunk is
// M=128 N=64 in one of two TMEM buffers.  TMEM: Q parts [0, 96), S buffers [128, 192), [192, 256);
// two CTAs per SM.
//
// Two passes over the keys (the same MMAs, so the scores are identical in both):
//   1. running max m and sum l of 2^(s * scale * log2 e - m);
//   2. p = 2^(x) / l with x = s * scale * log2 e - m, c = clip(p, 1e-9, 1) and
//      sum c log2 c, where log2 p = x - log2 l exactly, so only one exponential per element
//      (p <= 1 always: the row max contributes 2^0 to l).
// Row entropies H = -ln 2 * sum go to shared memory, and each 64-row half of the CTA writes the
// fp64 sum of its rows in row order into the same per-(b, h, 64-row tile) partial slots as the
// CUDA-core kernel, which probs_heads_kernel then sums per head in a fixed order.
#include "attn_common.cuh"
#include "sm100.cuh"

#include <cudaTypedefs.h>
#include <mutex>

XSAKE_DEFINE_DEVICE_ERROR(enttc)

namespace xsake {
namespace {

using namespace sm100;

constexpr int kEtThreads = 192;
constexpr int kEtStages = 4;
constexpr int kEtChunkBytes = 64 * 64 * 2;          // one bf16 part of a 64-key chunk
constexpr int kEtStageBytes = 3 * kEtChunkBytes;
constexpr uint32_t kEtTmemCols = 256;
constexpr uint32_t kEtQ = 0, kEtS = 128;             // TMEM columns: Q parts, S buffer 0 (buffer 1 at +64)
constexpr uint32_t kEtIdesc = idesc_bf16(128, 64, false);
constexpr float kEtClip = 1e-9f;

struct EtBars {
  uint64_t k_full[kEtStages], k_empty[kEtStages];
  uint64_t s_full[2], s_free[2];
  uint64_t q_ready;
  uint64_t drain;
};
constexpr int kEtOffBar = kEtStages * kEtStageBytes;
constexpr int kEtOffMisc = kEtOffBar + (int)sizeof(EtBars);
constexpr int kEtSmemBytes = kEtOffMisc + 64 + 128 * 8 + 1024;   // misc words, row entropies, alignment
static_assert(kEtSmemBytes <= 113 * 1024, "two CTAs per SM");

struct EtParams {
  const void* q;           // [B, H, S, 64] fp32 or bf16 (strides qs)
  int64_t qs[3];
  int B, H, S;
  int nparts;              // 3 (fp32 inputs) or 1 (bf16 inputs)
  int q_fp32;              // Q element type
  int k_split;             // 1: K parts in the split buffer [3][B*H][S64][64]; 0: K is the bf16 input
  float scale_log2;        // scale * log2(e)
  double* partial;         // entropy: [B * H * ceil(S / 64)]
  float* p_out;            // weights: [B, H, S, S] fp32
  // masked weights (xsake_attn_entropy): the plan's mask copy [Bm, Hm, nq, nq] and the causal cut
  int masked;
  const int32_t* plan;
  const uint8_t* mask;
  int Bm, Hm, bs, causal;
};

// ------------------------------------------------------------------------------ K split
// x (fp32, strided [B, H, S, 64]) -> three bf16 parts [3][B * H][S64][64], rows past S zero.
__global__ void __launch_bounds__(256) split3_kernel(const float* __restrict__ x, int64_t s0, int64_t s1, int64_t s2,
                                                     int B, int H, int S, int S64, __nv_bfloat16* __restrict__ out) {
  const int64_t n = (int64_t)B * H * S64 * 8;           // 8 columns of 8 elements a row
  const int64_t part = (int64_t)B * H * S64 * 64;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int c = (int)(i & 7);
    const int64_t row = i >> 3;                          // (b * H + h) * S64 + s
    const int s = (int)(row % S64);
    const int64_t bh = row / S64;
    const int b = (int)(bh / H), h = (int)(bh % H);
    float v[8];
    if (s < S) {
      const float4* src = reinterpret_cast<const float4*>(x + b * s0 + h * s1 + (int64_t)s * s2 + 8 * c);
      const float4 a = src[0], bq = src[1];
      v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = bq.x; v[5] = bq.y; v[6] = bq.z; v[7] = bq.w;
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = 0.f;
    }
    uint32_t w[3][4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float r0 = v[2 * j], r1 = v[2 * j + 1];
#pragma unroll
      for (int p = 0; p < 3; ++p) {
        const __nv_bfloat162 hb = __floats2bfloat162_rn(r0, r1);
        w[p][j] = *reinterpret_cast<const uint32_t*>(&hb);
        r0 -= __bfloat162float(hb.x);
        r1 -= __bfloat162float(hb.y);
      }
    }
#pragma unroll
    for (int p = 0; p < 3; ++p)
      *reinterpret_cast<uint4*>(out + p * part + row * 64 + 8 * c) = make_uint4(w[p][0], w[p][1], w[p][2], w[p][3]);
  }
}

// ------------------------------------------------------------------------------ main kernel
__device__ __forceinline__ void et_fail(volatile int* abort, int detail) {
  if (atomicExch((int*)abort, 1) == 0) record_device_error(DEV_ERR_TIMEOUT, detail);
}

// Row max of 64 values with four running 3-input maxes.
__device__ __forceinline__ float et_max64(const float* x) {
  float a[4] = {x[0], x[1], x[2], x[3]};
#pragma unroll
  for (int j = 2; j < 32; ++j) a[j & 3] = max3(a[j & 3], x[2 * j], x[2 * j + 1]);
  return fmaxf(fmaxf(a[0], a[1]), fmaxf(a[2], a[3]));
}

// The three bf16 parts of 2 * NW consecutive columns of a row as packed words (even column in
// the low half, the TMEM A-operand layout).
template <int NW>
__device__ __forceinline__ void split_words(const float* v, uint32_t (&w1)[NW], uint32_t (&w2)[NW],
                                            uint32_t (&w3)[NW]) {
#pragma unroll
  for (int j = 0; j < NW; ++j) {
    float r0 = v[2 * j], r1 = v[2 * j + 1];
    __nv_bfloat162 b = __floats2bfloat162_rn(r0, r1);
    w1[j] = *reinterpret_cast<const uint32_t*>(&b);
    r0 -= __bfloat162float(b.x);
    r1 -= __bfloat162float(b.y);
    b = __floats2bfloat162_rn(r0, r1);
    w2[j] = *reinterpret_cast<const uint32_t*>(&b);
    r0 -= __bfloat162float(b.x);
    r1 -= __bfloat162float(b.y);
    b = __floats2bfloat162_rn(r0, r1);
    w3[j] = *reinterpret_cast<const uint32_t*>(&b);
  }
}

// MODE kEtEntropy: per-tile entropy partials; kEtProbs: the weights themselves (pass 2 writes p).
constexpr int kEtEntropy = 0, kEtProbs = 1;

template <int MODE>
__global__ void __launch_bounds__(kEtThreads, 2)
entropy_tc_kernel(const __grid_constant__ CUtensorMap tmK, const EtParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  EtBars* bars = reinterpret_cast<EtBars*>(smem + kEtOffBar);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kEtOffMisc);
  volatile int* abort = reinterpret_cast<volatile int*>(smem + kEtOffMisc + 4);
  double* s_row = reinterpret_cast<double*>(smem + kEtOffMisc + 64);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bh = blockIdx.y, b = bh / p.H, h = bh % p.H;
  const int nk = (p.S + 63) / 64;
  const int nsteps = 2 * nk;

  volatile int* plan_ok = reinterpret_cast<volatile int*>(smem + kEtOffMisc + 8);
  if (threadIdx.x == 0) {
    *abort = 0;
    bool okp = true;
    if (p.masked) {
      const int32_t* hd = p.plan;
      okp = hd[H_MAGIC] == kPlanMagic && hd[H_VERSION] == kPlanVersion && hd[H_B] == p.B && hd[H_H] == p.H &&
            hd[H_S] == p.S && hd[H_BM] == p.Bm && hd[H_HM] == p.Hm && hd[H_BS] == p.bs && hd[H_CAUSAL] == p.causal;
      if (!okp) record_device_error(DEV_ERR_PLAN, 53);
    }
    *plan_ok = okp ? 1 : 0;
    for (int s = 0; s < kEtStages; ++s) {
      mbar_init(&bars->k_full[s], 1);
      mbar_init(&bars->k_empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bars->s_full[s], 1);
      mbar_init(&bars->s_free[s], 128);
    }
    mbar_init(&bars->q_ready, 128);
    mbar_init(&bars->drain, 1);
    fence_barrier_init();
  }
  if (warp == 4 && lane == 0) tma_prefetch_desc(&tmK);
  if (warp == 0) {
    tmem_alloc(tmem_slot, kEtTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (!*plan_ok) {
    if (MODE == kEtEntropy && threadIdx.x < 128 && (threadIdx.x & 63) == 0 && 2 * (int)blockIdx.x + (int)(threadIdx.x >> 6) < nk)
      p.partial[(int64_t)bh * nk + 2 * blockIdx.x + (threadIdx.x >> 6)] = (double)NAN;
  } else if (warp == 4) {
    // ------------------------------------------------------------------ K producer
    bool ok = true;
    for (int t = 0; t < nsteps && ok; ++t) {
      const int st = t % kEtStages, chunk = t % nk;
      if (!warp_mbar_wait(&bars->k_empty[st], ((t / kEtStages) & 1) ^ 1, abort)) { ok = false; break; }
      if (elect_one()) {
        uint8_t* buf = smem + st * kEtStageBytes;
        mbar_arrive_expect_tx(&bars->k_full[st], p.nparts * kEtChunkBytes);
        for (int q = 0; q < p.nparts; ++q)
          tma_load_4d(buf + q * kEtChunkBytes, &tmK, &bars->k_full[st], 0, 64 * chunk, p.k_split ? bh : h,
                      p.k_split ? q : b);
      }
      __syncwarp();
    }
    if (!ok && lane == 0) {
      et_fail(abort, 50);
      for (int s = 0; s < kEtStages; ++s) {   // bounded wait for copies in flight
        const uint64_t t0 = global_timer_ns();
        while (!mbar_try_wait(&bars->k_full[s], 0) && !mbar_try_wait(&bars->k_full[s], 1) &&
               global_timer_ns() - t0 < 1000000ull) {
        }
      }
    }
  } else if (warp == 5) {
    // ------------------------------------------------------------------ MMA issuer
    const uint64_t kdesc0 = sw128_desc(smem_u32(smem), 16, 1024);
    // products (Q part, K part), smallest first; bf16 inputs run only the last, q1 k1
    const int first = p.nparts == 3 ? 0 : 5;
    constexpr int kQi[6] = {2, 0, 1, 1, 0, 0}, kKj[6] = {0, 2, 1, 0, 1, 0};
    bool ok = warp_mbar_wait(&bars->q_ready, 0, abort);
    for (int t = 0; t < nsteps && ok; ++t) {
      const int st = t % kEtStages, buf = t & 1;
      if (!warp_mbar_wait2(&bars->k_full[st], (t / kEtStages) & 1, &bars->s_free[buf], ((t >> 1) & 1) ^ 1, t >= 2,
                           abort)) { ok = false; break; }
      tc_fence_after();
      if (elect_one()) {
        const uint32_t d = tmem + kEtS + 64 * buf;
#pragma unroll
        for (int pr = 0; pr < 6; ++pr) {
          if (pr < first) continue;
          const uint64_t kd = kdesc0 + (uint64_t)((st * kEtStageBytes + kKj[pr] * kEtChunkBytes) >> 4);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            mma_bf16_ts(d, tmem + kEtQ + 32 * kQi[pr] + 8 * kk, kd + 2 * kk, kEtIdesc,
                        (pr != first || kk) ? 1u : 0u);
        }
        mma_commit(&bars->s_full[buf]);
        mma_commit(&bars->k_empty[st]);
      }
      __syncwarp();
    }
    if (!ok && lane == 0) et_fail(abort, 51);
    if (elect_one()) mma_commit(&bars->drain);
    __syncwarp();
    if (lane == 0) {
      const uint64_t t0 = global_timer_ns();
      while (!mbar_try_wait(&bars->drain, 0) && global_timer_ns() - t0 < kWaitLimitNs) {
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------------ row threads
    const int r = threadIdx.x;                   // query row of the tile = TMEM lane
    const int tok = 128 * blockIdx.x + r;
    const bool valid = tok < p.S;
    const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
    // Q row -> TMEM: part i at columns [32 i, 32 i + 32), bf16 pair (2c, 2c + 1) in column c.
    if (p.q_fp32) {
      const float4* qr = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(p.q) + b * p.qs[0] +
                                                         h * p.qs[1] + (int64_t)(valid ? tok : 0) * p.qs[2]);
#pragma unroll
      for (int cb = 0; cb < 2; ++cb) {           // 32 columns at a time
        float v[32];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float4 x = valid ? qr[8 * cb + j] : make_float4(0.f, 0.f, 0.f, 0.f);
          v[4 * j] = x.x; v[4 * j + 1] = x.y; v[4 * j + 2] = x.z; v[4 * j + 3] = x.w;
        }
        uint32_t w1[16], w2[16], w3[16];
        split_words<16>(v, w1, w2, w3);
        XSAKE_TMEM_ST16(tmem + lane_base + kEtQ + 16 * cb, w1);
        XSAKE_TMEM_ST16(tmem + lane_base + kEtQ + 32 + 16 * cb, w2);
        XSAKE_TMEM_ST16(tmem + lane_base + kEtQ + 64 + 16 * cb, w3);
      }
    } else {
      const uint4* qr = reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(p.q) + b * p.qs[0] +
                                                       h * p.qs[1] + (int64_t)(valid ? tok : 0) * p.qs[2]);
      uint32_t w[32];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const uint4 x = valid ? qr[j] : make_uint4(0, 0, 0, 0);
        w[4 * j] = x.x; w[4 * j + 1] = x.y; w[4 * j + 2] = x.z; w[4 * j + 3] = x.w;
      }
      XSAKE_TMEM_ST32(tmem + lane_base + kEtQ, w);
    }
    tmem_wait_st();
    tc_fence_before();
    mbar_arrive(&bars->q_ready);

    constexpr float kClipTerm = -2.9897352853986263e-08f;   // 1e-9 * log2(1e-9)
    // A masked key's score in log2 units: its weight is 0 beside any live key and a row with no
    // live key comes out uniform, as finfo(float32).min does in the reference (finite, so that
    // m - m stays exact).
    constexpr float kFillLog2 = -1e30f;
    const uint64_t c2 = pk2(p.scale_log2, p.scale_log2);
    const uint8_t* mrow = nullptr;
    if (p.masked) {
      const int nq = p.S / p.bs;
      const int g = (p.Bm == 1 ? 0 : b) * p.Hm + (p.Hm == 1 ? 0 : h);
      mrow = p.mask + ((int64_t)g * nq + min(tok, p.S - 1) / p.bs) * nq;
    }
    // Masked keys of a chunk (block mask, causal cut) -> kFillLog2; keys past S are left to lim.
    auto mask_chunk = [&](float* x, int key0) {
      if (p.bs % 64 == 0) {
        const bool on = mrow[key0 / p.bs] != 0;
        const int cut = p.causal ? tok - key0 : 64;
#pragma unroll
        for (int j = 0; j < 64; ++j)
          if (!on || j > cut) x[j] = kFillLog2;
      } else {
        for (int j = 0; j < 64; ++j) {
          const int key = key0 + j;
          if (key < p.S && (!mrow[key / p.bs] || (p.causal && key > tok))) x[j] = kFillLog2;
        }
      }
    };
    float m = -INFINITY, l = 0.f, ent = 0.f, inv_l = 0.f, lg2l = 0.f;
    bool ok = true;
    // Pass-2 terms of one chunk: sum over its keys < lim of c log2 c (keys past the sequence
    // carry no weight and no clip term).
    auto terms = [&](const float* x, int lim, bool tail) {
      const uint64_t nm = pk2(-m, -m), il = pk2(inv_l, inv_l), nl = pk2(-lg2l, -lg2l);
      float a0 = 0.f, a1 = 0.f;
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const uint64_t d = add2(pk2(x[2 * j], x[2 * j + 1]), nm);
        float d0, d1;
        upk2(d, d0, d1);
        float p0, p1, l0, l1;
        upk2(mul2(pk2(ex2(d0), ex2(d1)), il), p0, p1);
        upk2(add2(d, nl), l0, l1);   // log2 p
        float t0 = p0 >= kEtClip ? p0 * fminf(l0, 0.f) : kClipTerm;
        float t1 = p1 >= kEtClip ? p1 * fminf(l1, 0.f) : kClipTerm;
        if (tail) {
          t0 = 2 * j < lim ? t0 : 0.f;
          t1 = 2 * j + 1 < lim ? t1 : 0.f;
        }
        a0 += t0;
        a1 += t1;
      }
      return a0 + a1;
    };
    // Pass-2 weights of one chunk of this row: p = 2^(x - m) / l for its keys < lim, written
    // 16 bytes at a time when rows start on 16-byte boundaries.
    auto store_probs = [&](const float* x, int lim, int chunk) {
      float* dst = p.p_out + ((int64_t)bh * p.S + tok) * p.S + 64 * chunk;
      const uint64_t nm = pk2(-m, -m), il = pk2(inv_l, inv_l);
      if (lim >= 64 && (p.S & 3) == 0) {
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          float d0, d1, d2, d3, p0, p1, p2, p3;
          upk2(add2(pk2(x[4 * j], x[4 * j + 1]), nm), d0, d1);
          upk2(add2(pk2(x[4 * j + 2], x[4 * j + 3]), nm), d2, d3);
          upk2(mul2(pk2(ex2(d0), ex2(d1)), il), p0, p1);
          upk2(mul2(pk2(ex2(d2), ex2(d3)), il), p2, p3);
          reinterpret_cast<float4*>(dst)[j] = make_float4(p0, p1, p2, p3);
        }
      } else {
#pragma unroll
        for (int j = 0; j < 64; ++j)
          if (j < lim) dst[j] = ex2(x[j] - m) * inv_l;
      }
    };
    for (int t = 0; t < nsteps; ++t) {
      const int buf = t & 1;
      if (!warp_mbar_wait(&bars->s_full[buf], (t >> 1) & 1, abort)) { ok = false; break; }
      tc_fence_after();
      uint32_t sr[64];
      XSAKE_TMEM_LD32(tmem + lane_base + kEtS + 64 * buf, sr);
      XSAKE_TMEM_LD32(tmem + lane_base + kEtS + 64 * buf + 32, (sr + 32));
      XSAKE_TMEM_WAIT_LD32(sr);
      XSAKE_TMEM_WAIT_LD32((sr + 32));
      tc_fence_before();
      mbar_arrive(&bars->s_free[buf]);            // the scores are in registers
      float* x = reinterpret_cast<float*>(sr);
      const int chunk = t < nk ? t : t - nk;
      const int lim = p.S - 64 * chunk;           // keys of the chunk inside the sequence (uniform)
#pragma unroll
      for (int j = 0; j < 32; ++j) upk2(mul2(pk2(x[2 * j], x[2 * j + 1]), c2), x[2 * j], x[2 * j + 1]);
      if (p.masked) mask_chunk(x, 64 * chunk);
      if (t < nk) {
        // pass 1: running max and sum (keys past the sequence are -inf)
        if (lim < 64) {
#pragma unroll
          for (int j = 0; j < 64; ++j)
            if (j >= lim) x[j] = -INFINITY;
        }
        const float mx = et_max64(x);
        if (mx > m) {
          l = (m == -INFINITY) ? 0.f : l * ex2(m - mx);
          m = mx;
        }
        const uint64_t nm = pk2(-m, -m);
        uint64_t acc[4] = {0ull, 0ull, 0ull, 0ull};
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          float e0, e1;
          upk2(add2(pk2(x[2 * j], x[2 * j + 1]), nm), e0, e1);
          acc[j & 3] = add2(acc[j & 3], pk2(ex2(e0), ex2(e1)));
        }
        float s0, s1;
        upk2(add2(add2(acc[0], acc[1]), add2(acc[2], acc[3])), s0, s1);
        l += s0 + s1;
        if (t == nk - 1) {
          inv_l = 1.f / l;
          lg2l = log2f(l);
        }
      } else if (MODE == kEtProbs) {
        if (valid) store_probs(x, lim, chunk);
      } else {
        ent += lim < 64 ? terms(x, lim, true) : terms(x, 64, false);
      }
    }
    // Row entropy H = -ln 2 * sum c log2 c; each 64-row half sums its rows in order in fp64.
    s_row[r] = !ok ? (double)NAN : valid ? -(double)(ent * kLn2) : 0.0;
    named_bar_sync(1, 128);
    if (MODE == kEtEntropy && (r & 63) == 0) {
      double acc = 0.0;
      for (int i = r; i < r + 64; ++i) acc += s_row[i];
      const int tile = 2 * blockIdx.x + (r >> 6);
      if (tile < nk) p.partial[(int64_t)bh * nk + tile] = acc;
    }
    if (!ok && r == 0) et_fail(abort, 52);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, kEtTmemCols);
  }
}

constexpr int kEtMaxDev = 64;
std::once_flag g_et_attr_once[kEtMaxDev];
cudaError_t g_et_attr_err[kEtMaxDev];

cudaError_t et_set_attributes() {
  cudaError_t e = cudaFuncSetAttribute(entropy_tc_kernel<kEtEntropy>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       kEtSmemBytes);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(entropy_tc_kernel<kEtProbs>, cudaFuncAttributeMaxDynamicSharedMemorySize, kEtSmemBytes);
  return e;
}

}  // namespace

size_t entropy_tc_split_bytes(int64_t batch, int64_t heads, int64_t seq) {
  return (size_t)3 * batch * heads * ((seq + 63) / 64 * 64) * 64 * 2;
}

// Launches the split (fp32 inputs) and the entropy kernel (of the masked weights when mask is
// given; writing the weights themselves to p_out instead when p_out is given); partial = [B * H * ceil(S / 64)] doubles,
// split_buf (fp32 inputs) = entropy_tc_split_bytes(B, H, S) bytes, 256-byte aligned.
int entropy_tc(int dtype, const void* q, const void* k, const int64_t qs[3], const int64_t ks[3], int B, int H,
               int S, float scale, double* partial, void* split_buf, cudaStream_t s, const EtMask* mask,
               float* p_out) {
  DeviceInfo di;
  int st = device_info(&di);
  if (st) return st;
  XSAKE_REQUIRE(di.major == 10, XSAKE_EUNSUPPORTED, "tensor-core entropy needs sm_100 (got sm_%d%d)", di.major,
                di.minor);
  const bool f32 = dtype == XSAKE_F32;
  const int64_t al = f32 ? 4 : 8;   // 16-byte rows and row starts
  XSAKE_REQUIRE(((uintptr_t)q & 15) == 0 && ((uintptr_t)k & 15) == 0 && qs[0] % al == 0 && qs[1] % al == 0 &&
                    qs[2] % al == 0 && ks[0] % al == 0 && ks[1] % al == 0 && ks[2] % al == 0,
                XSAKE_EINVAL, "q and k rows must be 16-byte aligned");
  const int S64 = (S + 63) / 64 * 64;
  CUtensorMap mk;
  if (f32) {
    XSAKE_REQUIRE(split_buf && ((uintptr_t)split_buf & 255) == 0, XSAKE_EINVAL, "split buffer must be 256-byte aligned");
    const int64_t n = (int64_t)B * H * S64 * 8;
    const int grid = (int)std::min<int64_t>((n + 255) / 256, (int64_t)di.sm_count * 8);
    split3_kernel<<<grid, 256, 0, s>>>(reinterpret_cast<const float*>(k), ks[0], ks[1], ks[2], B, H, S, S64,
                                       reinterpret_cast<__nv_bfloat16*>(split_buf));
    if ((st = check_launch("split3_kernel"))) return st;
    const int64_t sst[3] = {(int64_t)B * H * S64 * 64, (int64_t)S64 * 64, 64};
    if ((st = tc_make_map(&mk, split_buf, sst, 3, B * H, S64, 64))) return st;
  } else {
    if ((st = tc_make_map(&mk, k, ks, B, H, S, 64))) return st;
  }
  int dev = 0;
  XSAKE_CUDA_TRY(cudaGetDevice(&dev));
  XSAKE_REQUIRE(dev < kEtMaxDev, XSAKE_EUNSUPPORTED, "device ordinal %d", dev);
  std::call_once(g_et_attr_once[dev], [dev] { g_et_attr_err[dev] = et_set_attributes(); });
  XSAKE_REQUIRE(g_et_attr_err[dev] == cudaSuccess, XSAKE_ECUDA, "cudaFuncSetAttribute: %s",
                cudaGetErrorString(g_et_attr_err[dev]));
  EtParams p{};
  p.q = q;
  for (int i = 0; i < 3; ++i) p.qs[i] = qs[i];
  p.B = B;
  p.H = H;
  p.S = S;
  p.nparts = f32 ? 3 : 1;
  p.q_fp32 = f32 ? 1 : 0;
  p.k_split = f32 ? 1 : 0;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.partial = partial;
  if (mask) {
    p.masked = 1;
    p.plan = mask->plan;
    p.mask = mask->mask;
    p.Bm = mask->Bm;
    p.Hm = mask->Hm;
    p.bs = mask->bs;
    p.causal = mask->causal;
  }
  p.p_out = p_out;
  dim3 grid((S + 127) / 128, B * H);
  if (p_out) {
    XSAKE_REQUIRE(((uintptr_t)p_out & 15) == 0, XSAKE_EINVAL, "p must be 16-byte aligned");
    entropy_tc_kernel<kEtProbs><<<grid, kEtThreads, kEtSmemBytes, s>>>(mk, p);
  } else {
    entropy_tc_kernel<kEtEntropy><<<grid, kEtThreads, kEtSmemBytes, s>>>(mk, p);
  }
  return check_launch(p_out ? "entropy_tc_kernel (weights)" : "entropy_tc_kernel");
}

}  // namespace xsake
