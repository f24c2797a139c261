// Row kernels: softmax (fused_softmax, kernels/pallas/fused_softmax.py:26-87) and LayerNorm
// (fused_layernorm, kernels/pallas/fused_layernorm.py:26-119), forward and backward.
//
// HBM-bound single-pass design: one warp owns one row; the row is loaded once into registers
// with 16-byte coalesced loads (consecutive lanes, consecutive 16-byte words), reduced with
// warp shuffles and written once.  Statistics are fp32 whatever the storage dtype.  Rows too
// long for registers use a three-sweep fallback that re-reads the row (served from L1/L2).
#include "common.cuh"

#include <algorithm>
#include <math.h>

XSAKE_DEFINE_DEVICE_ERROR(rowops)

namespace xsake {
namespace {

// 16-byte vector of storage type T and its float expansion.
template <typename T> struct Vec;
template <> struct Vec<float> {
  static constexpr int N = 4;
  __device__ static void from_raw(const uint4& r, float* x) {
    x[0] = __uint_as_float(r.x); x[1] = __uint_as_float(r.y); x[2] = __uint_as_float(r.z); x[3] = __uint_as_float(r.w);
  }
  __device__ static void load(const void* p, float* x) {
    const float4 v = *reinterpret_cast<const float4*>(p);
    x[0] = v.x; x[1] = v.y; x[2] = v.z; x[3] = v.w;
  }
  __device__ static void store(void* p, const float* x) {
    *reinterpret_cast<float4*>(p) = make_float4(x[0], x[1], x[2], x[3]);
  }
};
template <> struct Vec<__nv_bfloat16> {
  static constexpr int N = 8;
  __device__ static void from_raw(const uint4& v, float* x) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const __nv_bfloat162 b = *reinterpret_cast<const __nv_bfloat162*>(&w[i]);
      x[2 * i] = __bfloat162float(b.x);
      x[2 * i + 1] = __bfloat162float(b.y);
    }
  }
  __device__ static void load(const void* p, float* x) {
    const uint4 v = *reinterpret_cast<const uint4*>(p);
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const __nv_bfloat162 b = *reinterpret_cast<const __nv_bfloat162*>(&w[i]);
      x[2 * i] = __bfloat162float(b.x);
      x[2 * i + 1] = __bfloat162float(b.y);
    }
  }
  __device__ static void store(void* p, const float* x) {
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      __nv_bfloat162 b = __floats2bfloat162_rn(x[2 * i], x[2 * i + 1]);
      w[i] = *reinterpret_cast<uint32_t*>(&b);
    }
    *reinterpret_cast<uint4*>(p) = make_uint4(w[0], w[1], w[2], w[3]);
  }
};

constexpr int kWarpsPerBlock = 8;

// ---------------------------------------------------------------------------------- softmax
template <typename T, int VPL>
__global__ void __launch_bounds__(256) softmax_fwd_reg(const T* __restrict__ x, T* __restrict__ y,
                                                       int64_t rows, int64_t cols) {
  constexpr int N = Vec<T>::N;
  const int lane = threadIdx.x & 31;
  const int64_t nvec = cols / N;
  for (int64_t row = (int64_t)blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5); row < rows;
       row += (int64_t)gridDim.x * kWarpsPerBlock) {
    const T* xr = x + row * cols;
    float v[VPL][N];
    float mx = -INFINITY;
#pragma unroll
    for (int k = 0; k < VPL; ++k) {
      const int64_t vi = lane + 32 * k;
      if (vi < nvec) {
        Vec<T>::load(xr + vi * N, v[k]);
      } else {
#pragma unroll
        for (int i = 0; i < N; ++i) v[k][i] = -INFINITY;
      }
#pragma unroll
      for (int i = 0; i < N; ++i) mx = fmaxf(mx, v[k][i]);
    }
    mx = warp_max(mx);
    float sum = 0.f;
#pragma unroll
    for (int k = 0; k < VPL; ++k)
#pragma unroll
      for (int i = 0; i < N; ++i) {
        v[k][i] = __expf(v[k][i] - mx);
        sum += v[k][i];
      }
    sum = warp_sum(sum);
    const float inv = 1.f / sum;
    T* yr = y + row * cols;
#pragma unroll
    for (int k = 0; k < VPL; ++k) {
      const int64_t vi = lane + 32 * k;
      if (vi < nvec) {
#pragma unroll
        for (int i = 0; i < N; ++i) v[k][i] *= inv;
        Vec<T>::store(yr + vi * N, v[k]);
      }
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(256) softmax_fwd_generic(const T* __restrict__ x, T* __restrict__ y,
                                                           int64_t rows, int64_t cols) {
  const int lane = threadIdx.x & 31;
  for (int64_t row = (int64_t)blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5); row < rows;
       row += (int64_t)gridDim.x * kWarpsPerBlock) {
    const T* xr = x + row * cols;
    float mx = -INFINITY;
    for (int64_t c = lane; c < cols; c += 32) mx = fmaxf(mx, DT<T>::to_f(xr[c]));
    mx = warp_max(mx);
    float sum = 0.f;
    for (int64_t c = lane; c < cols; c += 32) sum += __expf(DT<T>::to_f(xr[c]) - mx);
    sum = warp_sum(sum);
    const float inv = 1.f / sum;
    T* yr = y + row * cols;
    for (int64_t c = lane; c < cols; c += 32) yr[c] = DT<T>::from_f(__expf(DT<T>::to_f(xr[c]) - mx) * inv);
  }
}

template <typename T, int VPL>
__global__ void __launch_bounds__(256) softmax_bwd_reg(const T* __restrict__ y, const T* __restrict__ dy,
                                                       T* __restrict__ dx, int64_t rows, int64_t cols) {
  constexpr int N = Vec<T>::N;
  const int lane = threadIdx.x & 31;
  const int64_t nvec = cols / N;
  for (int64_t row = (int64_t)blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5); row < rows;
       row += (int64_t)gridDim.x * kWarpsPerBlock) {
    float yv[VPL][N], gv[VPL][N];
    float dot = 0.f;
#pragma unroll
    for (int k = 0; k < VPL; ++k) {
      const int64_t vi = lane + 32 * k;
      if (vi < nvec) {
        Vec<T>::load(y + row * cols + vi * N, yv[k]);
        Vec<T>::load(dy + row * cols + vi * N, gv[k]);
      } else {
#pragma unroll
        for (int i = 0; i < N; ++i) yv[k][i] = gv[k][i] = 0.f;
      }
#pragma unroll
      for (int i = 0; i < N; ++i) dot = fmaf(yv[k][i], gv[k][i], dot);
    }
    dot = warp_sum(dot);
#pragma unroll
    for (int k = 0; k < VPL; ++k) {
      const int64_t vi = lane + 32 * k;
      if (vi < nvec) {
        float o[N];
#pragma unroll
        for (int i = 0; i < N; ++i) o[i] = yv[k][i] * (gv[k][i] - dot);
        Vec<T>::store(dx + row * cols + vi * N, o);
      }
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(256) softmax_bwd_generic(const T* __restrict__ y, const T* __restrict__ dy,
                                                           T* __restrict__ dx, int64_t rows, int64_t cols) {
  const int lane = threadIdx.x & 31;
  for (int64_t row = (int64_t)blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5); row < rows;
       row += (int64_t)gridDim.x * kWarpsPerBlock) {
    const int64_t o = row * cols;
    float dot = 0.f;
    for (int64_t c = lane; c < cols; c += 32) dot += DT<T>::to_f(y[o + c]) * DT<T>::to_f(dy[o + c]);
    dot = warp_sum(dot);
    for (int64_t c = lane; c < cols; c += 32)
      dx[o + c] = DT<T>::from_f(DT<T>::to_f(y[o + c]) * (DT<T>::to_f(dy[o + c]) - dot));
  }
}

// ---------------------------------------------------------------------------------- layernorm
template <typename T, int VPL>
__global__ void __launch_bounds__(256) layernorm_fwd_reg(const T* __restrict__ x, const float* __restrict__ gamma,
                                                         const float* __restrict__ beta, float eps,
                                                         T* __restrict__ y, float* __restrict__ mean_out,
                                                         float* __restrict__ rstd_out, int64_t rows, int64_t d) {
  constexpr int N = Vec<T>::N;
  const int lane = threadIdx.x & 31;
  const int64_t nvec = d / N;
  const int64_t stride = (int64_t)gridDim.x * kWarpsPerBlock;
  int64_t row = (int64_t)blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5);
  // Rows are software-pipelined: the next row's 16-byte words are in flight while this row is
  // normalised, so each warp keeps two rows of loads outstanding.  The first row's loads are
  // issued before gamma/beta are staged so the two latencies overlap.
  uint4 nxt[VPL];
  auto fetch = [&](int64_t r) {
#pragma unroll
    for (int k = 0; k < VPL; ++k) {
      const int64_t vi = lane + 32 * k;
      nxt[k] = (r < rows && vi < nvec) ? *reinterpret_cast<const uint4*>(x + r * d + vi * N) : make_uint4(0, 0, 0, 0);
    }
  };
  fetch(row);
  // gamma/beta: read where each output is formed, 16 bytes at a time through the read-only L1
  // path (every warp of the SM reads the same 2 * d floats, so they stay in L1).  Measured
  // against staging them once per CTA in shared memory behind a CTA barrier: 7.6 vs 8.7 us at
  // bf16 [8192, 768], 21.4 vs 22.7 us at [32768, 768]; keeping them in registers would cost
  // 2 * VPL * N registers a thread and halve the resident warps.
  const float4* sg4 = reinterpret_cast<const float4*>(gamma);
  const float4* sb4 = reinterpret_cast<const float4*>(beta);
  const float inv_d = 1.f / (float)d;
  for (; row < rows; row += stride) {
    uint4 cur[VPL];
#pragma unroll
    for (int k = 0; k < VPL; ++k) cur[k] = nxt[k];
    fetch(row + stride);
    float v[VPL][N];
    float s = 0.f;
#pragma unroll
    for (int k = 0; k < VPL; ++k) {
      Vec<T>::from_raw(cur[k], v[k]);
#pragma unroll
      for (int i = 0; i < N; ++i) s += v[k][i];
    }
    const float mean = warp_sum(s) * inv_d;
    float q = 0.f;
#pragma unroll
    for (int k = 0; k < VPL; ++k) {
      const int64_t vi = lane + 32 * k;
#pragma unroll
      for (int i = 0; i < N; ++i) {
        const float c = (vi < nvec) ? v[k][i] - mean : 0.f;
        q = fmaf(c, c, q);
      }
    }
    const float var = warp_sum(q) * inv_d;
    const float rstd = 1.f / sqrtf(var + eps);
    T* yr = y + row * d;
#pragma unroll
    for (int k = 0; k < VPL; ++k) {
      const int64_t vi = lane + 32 * k;
      if (vi < nvec) {
        float o[N];
#pragma unroll
        for (int j = 0; j < N / 4; ++j) {
          const float4 g = __ldg(sg4 + vi * (N / 4) + j), b = __ldg(sb4 + vi * (N / 4) + j);
          o[4 * j + 0] = fmaf(g.x, (v[k][4 * j + 0] - mean) * rstd, b.x);
          o[4 * j + 1] = fmaf(g.y, (v[k][4 * j + 1] - mean) * rstd, b.y);
          o[4 * j + 2] = fmaf(g.z, (v[k][4 * j + 2] - mean) * rstd, b.z);
          o[4 * j + 3] = fmaf(g.w, (v[k][4 * j + 3] - mean) * rstd, b.w);
        }
        Vec<T>::store(yr + vi * N, o);
      }
    }
    if (lane == 0) {
      if (mean_out) mean_out[row] = mean;
      if (rstd_out) rstd_out[row] = rstd;
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(256) layernorm_fwd_generic(const T* __restrict__ x, const float* __restrict__ gamma,
                                                             const float* __restrict__ beta, float eps,
                                                             T* __restrict__ y, float* __restrict__ mean_out,
                                                             float* __restrict__ rstd_out, int64_t rows, int64_t d) {
  const int lane = threadIdx.x & 31;
  for (int64_t row = (int64_t)blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5); row < rows;
       row += (int64_t)gridDim.x * kWarpsPerBlock) {
    const T* xr = x + row * d;
    float s = 0.f;
    for (int64_t c = lane; c < d; c += 32) s += DT<T>::to_f(xr[c]);
    const float mean = warp_sum(s) / (float)d;
    float q = 0.f;
    for (int64_t c = lane; c < d; c += 32) {
      const float t = DT<T>::to_f(xr[c]) - mean;
      q = fmaf(t, t, q);
    }
    const float rstd = 1.f / sqrtf(warp_sum(q) / (float)d + eps);
    for (int64_t c = lane; c < d; c += 32)
      y[row * d + c] = DT<T>::from_f(fmaf(gamma[c], (DT<T>::to_f(xr[c]) - mean) * rstd, beta[c]));
    if (lane == 0) {
      if (mean_out) mean_out[row] = mean;
      if (rstd_out) rstd_out[row] = rstd;
    }
  }
}

// dx = rstd * (g*dy - mean(g*dy) - xhat * mean(g*dy*xhat)); per-CTA partial column sums of
// dy*xhat and dy go to `partial` [gridDim.x][2][d] and are reduced by ln_bwd_reduce.
template <typename T>
__global__ void __launch_bounds__(256) layernorm_bwd_rows(const T* __restrict__ x, const float* __restrict__ gamma,
                                                          const float* __restrict__ mean_in,
                                                          const float* __restrict__ rstd_in, const T* __restrict__ dy,
                                                          T* __restrict__ dx, float* __restrict__ partial,
                                                          int64_t rows, int64_t d) {
  extern __shared__ float sacc[];  // [2][d]
  for (int64_t c = threadIdx.x; c < 2 * d; c += blockDim.x) sacc[c] = 0.f;
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const float inv_d = 1.f / (float)d;
  // Rows are split into contiguous per-CTA ranges so the partial sums have a fixed order.
  const int64_t per = (rows + gridDim.x - 1) / gridDim.x;
  const int64_t r0 = (int64_t)blockIdx.x * per, r1 = min(rows, r0 + per);
  for (int64_t row = r0 + warp; row < r1; row += kWarpsPerBlock) {
    const int64_t o = row * d;
    const float mean = mean_in[row], rstd = rstd_in[row];
    float a1 = 0.f, a2 = 0.f;
    for (int64_t c = lane; c < d; c += 32) {
      const float xh = (DT<T>::to_f(x[o + c]) - mean) * rstd;
      const float gd = gamma[c] * DT<T>::to_f(dy[o + c]);
      a1 += gd;
      a2 = fmaf(gd, xh, a2);
    }
    a1 = warp_sum(a1) * inv_d;
    a2 = warp_sum(a2) * inv_d;
    for (int64_t c = lane; c < d; c += 32) {
      const float xh = (DT<T>::to_f(x[o + c]) - mean) * rstd;
      const float g = DT<T>::to_f(dy[o + c]);
      dx[o + c] = DT<T>::from_f(rstd * (gamma[c] * g - a1 - xh * a2));
    }
  }
  // Column partials: warps take turns in a fixed order (deterministic).
  for (int w = 0; w < kWarpsPerBlock; ++w) {
    if (warp == w) {
      for (int64_t row = r0 + warp; row < r1; row += kWarpsPerBlock) {
        const int64_t o = row * d;
        const float mean = mean_in[row], rstd = rstd_in[row];
        for (int64_t c = lane; c < d; c += 32) {
          const float g = DT<T>::to_f(dy[o + c]);
          sacc[c] = fmaf(g, (DT<T>::to_f(x[o + c]) - mean) * rstd, sacc[c]);
          sacc[d + c] += g;
        }
      }
    }
    __syncthreads();
  }
  for (int64_t c = threadIdx.x; c < 2 * d; c += blockDim.x) partial[(int64_t)blockIdx.x * 2 * d + c] = sacc[c];
}

// Register-resident backward for rows of 16-byte vectors: each warp owns whole rows (contiguous
// per-CTA ranges, as above), loads x and dy once with 16-byte loads, writes dx from registers and
// keeps its lanes' column partials (sum dy*xhat, sum dy) in registers across its rows; the CTA's
// warps are then summed in a fixed order, so the result stays deterministic.
template <typename T, int VPL>
__global__ void __launch_bounds__(256) layernorm_bwd_reg(const T* __restrict__ x, const float* __restrict__ gamma,
                                                         const float* __restrict__ mean_in,
                                                         const float* __restrict__ rstd_in, const T* __restrict__ dy,
                                                         T* __restrict__ dx, float* __restrict__ partial,
                                                         int64_t rows, int64_t d) {
  constexpr int N = Vec<T>::N;
  extern __shared__ float4 sm4[];
  float* sg = reinterpret_cast<float*>(sm4);   // gamma [d]
  float* wp = sg + d;                          // per-warp column partials [warps][2][d]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t nvec = d / N;
  for (int64_t c = threadIdx.x; c < d / 4; c += blockDim.x) sm4[c] = reinterpret_cast<const float4*>(gamma)[c];
  __syncthreads();
  const float4* sg4 = sm4;
  const float inv_d = 1.f / (float)d;
  const int64_t per = (rows + gridDim.x - 1) / gridDim.x;
  const int64_t r0 = (int64_t)blockIdx.x * per, r1 = min(rows, r0 + per);
  float cg[VPL][N], cb[VPL][N];
#pragma unroll
  for (int k = 0; k < VPL; ++k)
#pragma unroll
    for (int i = 0; i < N; ++i) cg[k][i] = cb[k][i] = 0.f;
  for (int64_t row = r0 + warp; row < r1; row += kWarpsPerBlock) {
    const float mean = mean_in[row], rstd = rstd_in[row];
    float xh[VPL][N], g[VPL][N];
#pragma unroll
    for (int k = 0; k < VPL; ++k) {
      const int64_t vi = lane + 32 * k;
      if (vi < nvec) {
        Vec<T>::load(x + row * d + vi * N, xh[k]);
        Vec<T>::load(dy + row * d + vi * N, g[k]);
      } else {
#pragma unroll
        for (int i = 0; i < N; ++i) xh[k][i] = g[k][i] = 0.f;
      }
    }
    float a1 = 0.f, a2 = 0.f;
#pragma unroll
    for (int k = 0; k < VPL; ++k) {
      const int64_t vi = lane + 32 * k;
      if (vi < nvec) {
#pragma unroll
        for (int j = 0; j < N / 4; ++j) {
          const float4 gm = sg4[vi * (N / 4) + j];
          const float gg[4] = {gm.x, gm.y, gm.z, gm.w};
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int i = 4 * j + q;
            xh[k][i] = (xh[k][i] - mean) * rstd;
            const float gd = gg[q] * g[k][i];
            a1 += gd;
            a2 = fmaf(gd, xh[k][i], a2);
            cg[k][i] = fmaf(g[k][i], xh[k][i], cg[k][i]);
            cb[k][i] += g[k][i];
          }
        }
      }
    }
    a1 = warp_sum(a1) * inv_d;
    a2 = warp_sum(a2) * inv_d;
#pragma unroll
    for (int k = 0; k < VPL; ++k) {
      const int64_t vi = lane + 32 * k;
      if (vi < nvec) {
        float o[N];
#pragma unroll
        for (int j = 0; j < N / 4; ++j) {
          const float4 gm = sg4[vi * (N / 4) + j];
          const float gg[4] = {gm.x, gm.y, gm.z, gm.w};
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int i = 4 * j + q;
            o[i] = rstd * (gg[q] * g[k][i] - a1 - xh[k][i] * a2);
          }
        }
        Vec<T>::store(dx + row * d + vi * N, o);
      }
    }
  }
#pragma unroll
  for (int k = 0; k < VPL; ++k) {
    const int64_t vi = lane + 32 * k;
    if (vi < nvec) {
#pragma unroll
      for (int i = 0; i < N; ++i) {
        wp[(int64_t)(2 * warp) * d + vi * N + i] = cg[k][i];
        wp[(int64_t)(2 * warp + 1) * d + vi * N + i] = cb[k][i];
      }
    }
  }
  __syncthreads();
  for (int64_t c = threadIdx.x; c < 2 * d; c += blockDim.x) {
    float acc = 0.f;
#pragma unroll
    for (int w = 0; w < kWarpsPerBlock; ++w) acc += wp[(int64_t)w * 2 * d + c];
    partial[(int64_t)blockIdx.x * 2 * d + c] = acc;
  }
}

// Sum of the per-CTA column partials: a CTA per 32 columns, warp w adds partial rows w, w+8, ...
// (lane = column, coalesced), then the 8 warp sums are added in order: fixed order throughout.
__global__ void __launch_bounds__(256) ln_bwd_reduce(const float* __restrict__ partial, int nblocks, int64_t d,
                                                     float* __restrict__ dgamma, float* __restrict__ dbeta) {
  __shared__ float ws[kWarpsPerBlock][32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t c = (int64_t)blockIdx.x * 32 + lane;
  float acc = 0.f;
  if (c < 2 * d) {
#pragma unroll 4
    for (int b = warp; b < nblocks; b += kWarpsPerBlock) acc += partial[(int64_t)b * 2 * d + c];
  }
  ws[warp][lane] = acc;
  __syncthreads();
  if (warp == 0 && c < 2 * d) {
    float t = 0.f;
#pragma unroll
    for (int w = 0; w < kWarpsPerBlock; ++w) t += ws[w][lane];
    if (c < d) dgamma[c] = t; else dbeta[c - d] = t;
  }
}

// ------------------------------------------------------------------------------ cross entropy
// cross_entropy_loss of model/transformer.py:177-203 over rows of logits (the vocabulary in the
// last axis, `ld` elements between rows, ld >= vocab).  One warp per row.  Forward: online max /
// sum of exp in fp32 from the logits' own dtype, lse = max + log(sum), nll = lse - logit[target]
// (0 for a target equal to ignore_index).  Backward: grad = coef * (softmax - onehot(target)) for
// the vocab columns and 0 for columns [vocab, ld) and for ignored rows, written over the whole
// row so the gradient buffer needs no fill.  coef (a device scalar) is d(loss)/d(sum of nll).
template <typename T, bool VEC>
__global__ void __launch_bounds__(256) xent_fwd_kernel(const T* __restrict__ logits, int64_t rows, int64_t vocab,
                                                       int64_t ld, const int64_t* __restrict__ targets,
                                                       int64_t ignore_index, float* __restrict__ lse_out,
                                                       float* __restrict__ nll_out) {
  constexpr int N = Vec<T>::N;
  constexpr float kL2e = 1.4426950408889634f;
  const int lane = threadIdx.x & 31;
  for (int64_t row = (int64_t)blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5); row < rows;
       row += (int64_t)gridDim.x * kWarpsPerBlock) {
    const T* r = logits + row * ld;
    float m = -INFINITY, sum = 0.f;
    auto add = [&](const float* v, int n) {
      float mv = v[0];
      for (int i = 1; i < n; ++i) mv = fmaxf(mv, v[i]);
      if (mv > m) {
        sum = m == -INFINITY ? 0.f : sum * exp2f((m - mv) * kL2e);
        m = mv;
      }
      if (m != -INFINITY)
        for (int i = 0; i < n; ++i) sum += exp2f((v[i] - m) * kL2e);
    };
    int64_t c0 = 0;
    if (VEC) {
      const int64_t nv = vocab / N;
      // Four 16-byte loads a lane in flight per round (the rows are ~100 KB: the loop is bound by
      // memory-level parallelism, not arithmetic).
      int64_t vi = lane;
      for (; vi + 96 < nv; vi += 128) {
        uint4 raw[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) raw[u] = *reinterpret_cast<const uint4*>(r + (vi + 32 * u) * N);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          float v[N];
          Vec<T>::from_raw(raw[u], v);
          add(v, N);
        }
      }
      for (; vi < nv; vi += 32) {
        float v[N];
        Vec<T>::load(r + vi * N, v);
        add(v, N);
      }
      c0 = nv * N;
    }
    for (int64_t c = c0 + lane; c < vocab; c += 32) {
      const float v = DT<T>::to_f(r[c]);
      add(&v, 1);
    }
    // Combine the lanes' (max, sum) pairs.
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const float mo = __shfl_xor_sync(0xffffffffu, m, off), so = __shfl_xor_sync(0xffffffffu, sum, off);
      const float mn = fmaxf(m, mo);
      sum = (m == -INFINITY ? 0.f : sum * exp2f((m - mn) * kL2e)) +
            (mo == -INFINITY ? 0.f : so * exp2f((mo - mn) * kL2e));
      m = mn;
    }
    if (lane == 0) {
      const float lse = m + logf(sum);
      const int64_t t = targets[row];
      const bool valid = t != ignore_index;
      const int64_t tc = t < 0 ? 0 : (t >= vocab ? vocab - 1 : t);
      lse_out[row] = lse;
      nll_out[row] = valid ? lse - DT<T>::to_f(r[tc]) : 0.f;
    }
  }
}

template <typename T, bool VEC>
__global__ void __launch_bounds__(256) xent_bwd_kernel(const T* __restrict__ logits, int64_t rows, int64_t vocab,
                                                       int64_t ld, const int64_t* __restrict__ targets,
                                                       int64_t ignore_index, const float* __restrict__ lse_in,
                                                       const float* __restrict__ coef, T* __restrict__ grad) {
  constexpr int N = Vec<T>::N;
  constexpr float kL2e = 1.4426950408889634f;
  const int lane = threadIdx.x & 31;
  const float cf = *coef;
  for (int64_t row = (int64_t)blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5); row < rows;
       row += (int64_t)gridDim.x * kWarpsPerBlock) {
    const T* r = logits + row * ld;
    T* gr = grad + row * ld;
    const int64_t t = targets[row];
    const bool valid = t != ignore_index;
    const int64_t tc = t < 0 ? 0 : (t >= vocab ? vocab - 1 : t);
    const float nl = -lse_in[row] * kL2e;
    const float c = valid ? cf : 0.f;
    auto g_of = [&](int64_t col, float x) {
      if (col >= vocab) return 0.f;
      return c * (exp2f(fmaf(x, kL2e, nl)) - (col == tc ? 1.f : 0.f));
    };
    int64_t c0 = 0;
    if (VEC) {
      const int64_t nv = ld / N;   // whole rows of vectors: ld % N == 0
      const int64_t nfull = vocab / N;   // vectors entirely inside the vocabulary
      int64_t vi = lane;
      // Four 16-byte loads a lane in flight per round over the vectors inside the vocabulary.
      for (; vi + 96 < nfull; vi += 128) {
        uint4 raw[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) raw[u] = *reinterpret_cast<const uint4*>(r + (vi + 32 * u) * N);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          float v[N], o[N];
          Vec<T>::from_raw(raw[u], v);
#pragma unroll
          for (int i = 0; i < N; ++i) o[i] = g_of((vi + 32 * u) * N + i, v[i]);
          Vec<T>::store(gr + (vi + 32 * u) * N, o);
        }
      }
      for (; vi < nv; vi += 32) {
        float v[N], o[N];
        if ((vi + 1) * N <= vocab) {
          Vec<T>::load(r + vi * N, v);
        } else {
#pragma unroll
          for (int i = 0; i < N; ++i) v[i] = vi * N + i < vocab ? DT<T>::to_f(r[vi * N + i]) : 0.f;
        }
#pragma unroll
        for (int i = 0; i < N; ++i) o[i] = g_of(vi * N + i, v[i]);
        Vec<T>::store(gr + vi * N, o);
      }
      c0 = nv * N;
    }
    for (int64_t col = c0 + lane; col < ld; col += 32)
      gr[col] = DT<T>::from_f(g_of(col, col < vocab ? DT<T>::to_f(r[col]) : 0.f));
  }
}

int grid_for_rows(int64_t rows, int sm_count, int ctas_per_sm = 32) {
  const int64_t blocks = (rows + kWarpsPerBlock - 1) / kWarpsPerBlock;
  return (int)std::max<int64_t>(1, std::min<int64_t>(blocks, (int64_t)sm_count * ctas_per_sm));
}

template <typename T>
int softmax_fwd_t(int64_t rows, int64_t cols, const void* x, void* y, cudaStream_t s, int sms) {
  constexpr int N = Vec<T>::N;
  const T* xp = reinterpret_cast<const T*>(x);
  T* yp = reinterpret_cast<T*>(y);
  const int grid = grid_for_rows(rows, sms);
  const bool vec_ok = cols % N == 0 && ((uintptr_t)x & 15) == 0 && ((uintptr_t)y & 15) == 0;
  const int64_t per_lane = (cols / N + 31) / 32;
  if (vec_ok && per_lane <= 1) softmax_fwd_reg<T, 1><<<grid, 256, 0, s>>>(xp, yp, rows, cols);
  else if (vec_ok && per_lane <= 2) softmax_fwd_reg<T, 2><<<grid, 256, 0, s>>>(xp, yp, rows, cols);
  else if (vec_ok && per_lane <= 4) softmax_fwd_reg<T, 4><<<grid, 256, 0, s>>>(xp, yp, rows, cols);
  else if (vec_ok && per_lane <= 8) softmax_fwd_reg<T, 8><<<grid, 256, 0, s>>>(xp, yp, rows, cols);
  else if (vec_ok && per_lane <= 16) softmax_fwd_reg<T, 16><<<grid, 256, 0, s>>>(xp, yp, rows, cols);
  else softmax_fwd_generic<T><<<grid, 256, 0, s>>>(xp, yp, rows, cols);
  return check_launch("softmax_fwd");
}

template <typename T>
int softmax_bwd_t(int64_t rows, int64_t cols, const void* y, const void* dy, void* dx, cudaStream_t s, int sms) {
  constexpr int N = Vec<T>::N;
  const T* yp = reinterpret_cast<const T*>(y);
  const T* gp = reinterpret_cast<const T*>(dy);
  T* dp = reinterpret_cast<T*>(dx);
  const int grid = grid_for_rows(rows, sms);
  const bool vec_ok = cols % N == 0 && (((uintptr_t)y | (uintptr_t)dy | (uintptr_t)dx) & 15) == 0;
  const int64_t per_lane = (cols / N + 31) / 32;
  if (vec_ok && per_lane <= 2) softmax_bwd_reg<T, 2><<<grid, 256, 0, s>>>(yp, gp, dp, rows, cols);
  else if (vec_ok && per_lane <= 4) softmax_bwd_reg<T, 4><<<grid, 256, 0, s>>>(yp, gp, dp, rows, cols);
  else if (vec_ok && per_lane <= 8) softmax_bwd_reg<T, 8><<<grid, 256, 0, s>>>(yp, gp, dp, rows, cols);
  else softmax_bwd_generic<T><<<grid, 256, 0, s>>>(yp, gp, dp, rows, cols);
  return check_launch("softmax_bwd");
}

template <typename T>
int layernorm_fwd_t(int64_t rows, int64_t d, const void* x, const float* g, const float* b, float eps, void* y,
                    float* mean, float* rstd, cudaStream_t s, int sms) {
  constexpr int N = Vec<T>::N;
  const T* xp = reinterpret_cast<const T*>(x);
  T* yp = reinterpret_cast<T*>(y);
  const bool vec_ok = d % N == 0 && d % 4 == 0 && (((uintptr_t)x | (uintptr_t)y | (uintptr_t)g | (uintptr_t)b) & 15) == 0;
  const int64_t per_lane = (d / N + 31) / 32;
  const size_t smem = 0;
  // One wave: as many CTAs as fit on the GPU at once, each warp normalising rows/grid rows.
  auto launch = [&](auto kern, size_t sm) {
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, 256, sm) != cudaSuccess || per_sm < 1) {
      (void)cudaGetLastError();
      per_sm = 2;
    }
    kern<<<grid_for_rows(rows, sms, per_sm), 256, sm, s>>>(xp, g, b, eps, yp, mean, rstd, rows, d);
  };
  if (vec_ok && per_lane <= 1) launch(layernorm_fwd_reg<T, 1>, smem);
  else if (vec_ok && per_lane <= 2) launch(layernorm_fwd_reg<T, 2>, smem);
  else if (vec_ok && per_lane <= 3) launch(layernorm_fwd_reg<T, 3>, smem);
  else if (vec_ok && per_lane <= 4) launch(layernorm_fwd_reg<T, 4>, smem);
  else if (vec_ok && per_lane <= 8) launch(layernorm_fwd_reg<T, 8>, smem);
  else layernorm_fwd_generic<T><<<grid_for_rows(rows, sms, 8), 256, 0, s>>>(xp, g, b, eps, yp, mean, rstd, rows, d);
  return check_launch("layernorm_fwd");
}

int ln_bwd_blocks(int64_t rows, int sms) {
  return (int)std::max<int64_t>(1, std::min<int64_t>((rows + 31) / 32, (int64_t)sms * 4));
}

}  // namespace
}  // namespace xsake

using namespace xsake;

static int check_dtype(int32_t dt) {
  XSAKE_REQUIRE(dt == XSAKE_F32 || dt == XSAKE_BF16, XSAKE_EINVAL, "dtype %d", dt);
  return XSAKE_OK;
}

extern "C" int xsake_softmax_fwd(int32_t dtype, int64_t rows, int64_t cols, const void* x_dev, void* y_dev,
                                 void* stream) {
  clear_error();
  int st = check_dtype(dtype);
  if (st) return st;
  XSAKE_REQUIRE(rows >= 0 && cols > 0, XSAKE_EINVAL, "rows must be >= 0 and cols > 0");
  if (rows == 0) return XSAKE_OK;
  XSAKE_REQUIRE(x_dev && y_dev, XSAKE_EINVAL, "NULL pointer");
  DeviceInfo di;
  if ((st = device_info(&di))) return st;
  return dtype == XSAKE_F32 ? softmax_fwd_t<float>(rows, cols, x_dev, y_dev, as_stream(stream), di.sm_count)
                            : softmax_fwd_t<__nv_bfloat16>(rows, cols, x_dev, y_dev, as_stream(stream), di.sm_count);
}

extern "C" int xsake_softmax_bwd(int32_t dtype, int64_t rows, int64_t cols, const void* y_dev, const void* dy_dev,
                                 void* dx_dev, void* stream) {
  clear_error();
  int st = check_dtype(dtype);
  if (st) return st;
  XSAKE_REQUIRE(rows >= 0 && cols > 0, XSAKE_EINVAL, "rows must be >= 0 and cols > 0");
  if (rows == 0) return XSAKE_OK;
  XSAKE_REQUIRE(y_dev && dy_dev && dx_dev, XSAKE_EINVAL, "NULL pointer");
  DeviceInfo di;
  if ((st = device_info(&di))) return st;
  return dtype == XSAKE_F32
             ? softmax_bwd_t<float>(rows, cols, y_dev, dy_dev, dx_dev, as_stream(stream), di.sm_count)
             : softmax_bwd_t<__nv_bfloat16>(rows, cols, y_dev, dy_dev, dx_dev, as_stream(stream), di.sm_count);
}

extern "C" int xsake_layernorm_fwd(int32_t x_dtype, int64_t rows, int64_t d, const void* x_dev,
                                   const float* gamma_dev, const float* beta_dev, float eps, void* y_dev,
                                   float* mean_dev, float* rstd_dev, void* stream) {
  clear_error();
  int st = check_dtype(x_dtype);
  if (st) return st;
  XSAKE_REQUIRE(rows >= 0 && d > 0, XSAKE_EINVAL, "rows must be >= 0 and d > 0");
  XSAKE_REQUIRE(eps >= 0.f, XSAKE_EINVAL, "eps must be >= 0");
  if (rows == 0) return XSAKE_OK;
  XSAKE_REQUIRE(x_dev && gamma_dev && beta_dev && y_dev, XSAKE_EINVAL, "NULL pointer");
  DeviceInfo di;
  if ((st = device_info(&di))) return st;
  cudaStream_t s = as_stream(stream);
  return x_dtype == XSAKE_F32
             ? layernorm_fwd_t<float>(rows, d, x_dev, gamma_dev, beta_dev, eps, y_dev, mean_dev, rstd_dev, s, di.sm_count)
             : layernorm_fwd_t<__nv_bfloat16>(rows, d, x_dev, gamma_dev, beta_dev, eps, y_dev, mean_dev, rstd_dev, s,
                                              di.sm_count);
}

extern "C" int xsake_layernorm_bwd_workspace_size(int64_t rows, int64_t d, size_t* bytes) {
  clear_error();
  XSAKE_REQUIRE(bytes != nullptr && rows >= 0 && d > 0, XSAKE_EINVAL, "bad arguments");
  DeviceInfo di;
  int st = device_info(&di);
  const int sms = st ? 148 : di.sm_count;
  clear_error();
  *bytes = (size_t)ln_bwd_blocks(rows, sms) * 2 * (size_t)d * sizeof(float);
  return XSAKE_OK;
}

extern "C" int xsake_layernorm_bwd(int32_t x_dtype, int64_t rows, int64_t d, const void* x_dev,
                                   const float* gamma_dev, const float* mean_dev, const float* rstd_dev,
                                   const void* dy_dev, void* dx_dev, float* dgamma_dev, float* dbeta_dev,
                                   void* workspace_dev, size_t workspace_bytes, void* stream) {
  clear_error();
  int st = check_dtype(x_dtype);
  if (st) return st;
  XSAKE_REQUIRE(rows > 0 && d > 0, XSAKE_EINVAL, "rows and d must be positive");
  XSAKE_REQUIRE(x_dev && gamma_dev && mean_dev && rstd_dev && dy_dev && dx_dev && dgamma_dev && dbeta_dev,
                XSAKE_EINVAL, "NULL pointer");
  XSAKE_REQUIRE(2 * d * sizeof(float) <= 96 * 1024, XSAKE_EUNSUPPORTED, "d too large for the backward");
  DeviceInfo di;
  if ((st = device_info(&di))) return st;
  const int nb = ln_bwd_blocks(rows, di.sm_count);
  XSAKE_REQUIRE(workspace_dev && workspace_bytes >= (size_t)nb * 2 * d * sizeof(float), XSAKE_EINVAL,
                "workspace too small");
  cudaStream_t s = as_stream(stream);
  const size_t smem = 2 * d * sizeof(float);
  float* partial = reinterpret_cast<float*>(workspace_dev);
  // Rows of whole 16-byte vectors, up to 6 (fp32) or 4 (bf16) vectors a lane (d <= 768 fp32,
  // d <= 1024 bf16; wider rows would spill): the register-resident kernel.
  const int nvec_lane = x_dtype == XSAKE_F32 ? (int)((d / 4 + 31) / 32) : (int)((d / 8 + 31) / 32);
  const bool vec_ok = d % 8 == 0 && ((uintptr_t)x_dev & 15) == 0 && ((uintptr_t)dy_dev & 15) == 0 &&
                      ((uintptr_t)dx_dev & 15) == 0 && ((uintptr_t)gamma_dev & 15) == 0 &&
                      nvec_lane <= (x_dtype == XSAKE_F32 ? 6 : 4);
  const size_t smem_reg = (size_t)(1 + 2 * kWarpsPerBlock) * d * sizeof(float);
  if (vec_ok && smem_reg <= 200 * 1024) {
    auto launch = [&](auto kern, auto xp, auto dyp, auto dxp) -> int {
      XSAKE_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_reg));
      kern<<<nb, 256, smem_reg, s>>>(xp, gamma_dev, mean_dev, rstd_dev, dyp, dxp, partial, rows, d);
      return check_launch("layernorm_bwd_reg");
    };
    if (x_dtype == XSAKE_F32) {
      const float* xp = (const float*)x_dev;
      const float* dyp = (const float*)dy_dev;
      float* dxp = (float*)dx_dev;
      if (nvec_lane <= 2) st = launch(layernorm_bwd_reg<float, 2>, xp, dyp, dxp);
      else if (nvec_lane <= 4) st = launch(layernorm_bwd_reg<float, 4>, xp, dyp, dxp);
      else st = launch(layernorm_bwd_reg<float, 6>, xp, dyp, dxp);
    } else {
      const __nv_bfloat16* xp = (const __nv_bfloat16*)x_dev;
      const __nv_bfloat16* dyp = (const __nv_bfloat16*)dy_dev;
      __nv_bfloat16* dxp = (__nv_bfloat16*)dx_dev;
      if (nvec_lane <= 1) st = launch(layernorm_bwd_reg<__nv_bfloat16, 1>, xp, dyp, dxp);
      else if (nvec_lane <= 2) st = launch(layernorm_bwd_reg<__nv_bfloat16, 2>, xp, dyp, dxp);
      else if (nvec_lane <= 3) st = launch(layernorm_bwd_reg<__nv_bfloat16, 3>, xp, dyp, dxp);
      else st = launch(layernorm_bwd_reg<__nv_bfloat16, 4>, xp, dyp, dxp);
    }
    if (st) return st;
    ln_bwd_reduce<<<(int)((2 * d + 31) / 32), 256, 0, s>>>(partial, nb, d, dgamma_dev, dbeta_dev);
    return check_launch("ln_bwd_reduce");
  }
  if (x_dtype == XSAKE_F32) {
    if (smem > 48 * 1024)
      XSAKE_CUDA_TRY(cudaFuncSetAttribute(layernorm_bwd_rows<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    layernorm_bwd_rows<float><<<nb, 256, smem, s>>>((const float*)x_dev, gamma_dev, mean_dev, rstd_dev,
                                                    (const float*)dy_dev, (float*)dx_dev, partial, rows, d);
  } else {
    if (smem > 48 * 1024)
      XSAKE_CUDA_TRY(cudaFuncSetAttribute(layernorm_bwd_rows<__nv_bfloat16>,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    layernorm_bwd_rows<__nv_bfloat16><<<nb, 256, smem, s>>>(
        (const __nv_bfloat16*)x_dev, gamma_dev, mean_dev, rstd_dev, (const __nv_bfloat16*)dy_dev,
        (__nv_bfloat16*)dx_dev, partial, rows, d);
  }
  if ((st = check_launch("layernorm_bwd_rows"))) return st;
  ln_bwd_reduce<<<(int)((2 * d + 31) / 32), 256, 0, s>>>(partial, nb, d, dgamma_dev, dbeta_dev);
  return check_launch("ln_bwd_reduce");
}

extern "C" int xsake_xent_fwd(int32_t dtype, int64_t rows, int64_t vocab, int64_t ld, const void* logits_dev,
                              const int64_t* targets_dev, int64_t ignore_index, float* lse_dev, float* nll_dev,
                              void* stream) {
  clear_error();
  int st = check_dtype(dtype);
  if (st) return st;
  XSAKE_REQUIRE(rows >= 0 && vocab > 0 && ld >= vocab, XSAKE_EINVAL, "need rows >= 0, vocab > 0, ld >= vocab");
  if (rows == 0) return XSAKE_OK;
  XSAKE_REQUIRE(logits_dev && targets_dev && lse_dev && nll_dev, XSAKE_EINVAL, "NULL pointer");
  DeviceInfo di;
  if ((st = device_info(&di))) return st;
  cudaStream_t s = as_stream(stream);
  const int grid = grid_for_rows(rows, di.sm_count, 8);
  const bool vec = ld % 8 == 0 && ((uintptr_t)logits_dev & 15) == 0;
  if (dtype == XSAKE_F32) {
    const float* x = (const float*)logits_dev;
    if (vec) xent_fwd_kernel<float, true><<<grid, 256, 0, s>>>(x, rows, vocab, ld, targets_dev, ignore_index, lse_dev, nll_dev);
    else xent_fwd_kernel<float, false><<<grid, 256, 0, s>>>(x, rows, vocab, ld, targets_dev, ignore_index, lse_dev, nll_dev);
  } else {
    const __nv_bfloat16* x = (const __nv_bfloat16*)logits_dev;
    if (vec) xent_fwd_kernel<__nv_bfloat16, true><<<grid, 256, 0, s>>>(x, rows, vocab, ld, targets_dev, ignore_index, lse_dev, nll_dev);
    else xent_fwd_kernel<__nv_bfloat16, false><<<grid, 256, 0, s>>>(x, rows, vocab, ld, targets_dev, ignore_index, lse_dev, nll_dev);
  }
  return check_launch("xent_fwd_kernel");
}

extern "C" int xsake_xent_bwd(int32_t dtype, int64_t rows, int64_t vocab, int64_t ld, const void* logits_dev,
                              const int64_t* targets_dev, int64_t ignore_index, const float* lse_dev,
                              const float* coef_dev, void* grad_dev, void* stream) {
  clear_error();
  int st = check_dtype(dtype);
  if (st) return st;
  XSAKE_REQUIRE(rows >= 0 && vocab > 0 && ld >= vocab, XSAKE_EINVAL, "need rows >= 0, vocab > 0, ld >= vocab");
  if (rows == 0) return XSAKE_OK;
  XSAKE_REQUIRE(logits_dev && targets_dev && lse_dev && coef_dev && grad_dev, XSAKE_EINVAL, "NULL pointer");
  DeviceInfo di;
  if ((st = device_info(&di))) return st;
  cudaStream_t s = as_stream(stream);
  const int grid = grid_for_rows(rows, di.sm_count, 8);
  const bool vec = ld % 8 == 0 && ((uintptr_t)logits_dev & 15) == 0 && ((uintptr_t)grad_dev & 15) == 0;
  if (dtype == XSAKE_F32) {
    const float* x = (const float*)logits_dev;
    float* g = (float*)grad_dev;
    if (vec) xent_bwd_kernel<float, true><<<grid, 256, 0, s>>>(x, rows, vocab, ld, targets_dev, ignore_index, lse_dev, coef_dev, g);
    else xent_bwd_kernel<float, false><<<grid, 256, 0, s>>>(x, rows, vocab, ld, targets_dev, ignore_index, lse_dev, coef_dev, g);
  } else {
    const __nv_bfloat16* x = (const __nv_bfloat16*)logits_dev;
    __nv_bfloat16* g = (__nv_bfloat16*)grad_dev;
    if (vec) xent_bwd_kernel<__nv_bfloat16, true><<<grid, 256, 0, s>>>(x, rows, vocab, ld, targets_dev, ignore_index, lse_dev, coef_dev, g);
    else xent_bwd_kernel<__nv_bfloat16, false><<<grid, 256, 0, s>>>(x, rows, vocab, ld, targets_dev, ignore_index, lse_dev, coef_dev, g);
  }
  return check_launch("xent_bwd_kernel");
}
