// CUDA-core (SIMT) attention kernels: the fp32 path (where tensor-core precision would not
// meet a 1e-5 tolerance), any block size, head_dim in {16, 32, 64, 128}, and the backward.
//
// Semantics follow sparse_attention_reference (kernels/pallas/sparse_attention.py:45-91):
// a score is live when its block is on in the mask and, if causal, key <= query; the row
// softmax runs over live scores; a row with no live score attends uniformly to all S keys
// (the reference fills masked scores with finfo.min).  The backward is autodiff of that
// function: masked scores pass no gradient, so fully masked rows only feed dV.
#include "attn_common.cuh"

#include <math.h>

XSAKE_DEFINE_DEVICE_ERROR(simt)

namespace xsake {
namespace {

constexpr int kQT = 64;   // query rows per CTA (two threads per row)
constexpr int kKT = 32;   // key rows per shared-memory tile

template <typename T>
__device__ __forceinline__ float ld(const void* p, int64_t i) {
  return DT<T>::to_f(reinterpret_cast<const T*>(p)[i]);
}
template <typename T>
__device__ __forceinline__ void st(void* p, int64_t i, float x) {
  reinterpret_cast<T*>(p)[i] = DT<T>::from_f(x);
}

__device__ __forceinline__ const uint8_t* group_mask(const AttnArgs& a, int b, int h) {
  const uint8_t* m = reinterpret_cast<const uint8_t*>(a.plan + a.L.mask_off);
  return m + (int64_t)a.L.group_of(b, h) * a.L.nq * a.L.nq;
}

// True when any (query in [q0,q1], key in [k0,k1]) pair can be live (block level + causal).
__device__ __forceinline__ bool tile_live(const AttnArgs& a, const uint8_t* m, int q0, int q1, int k0, int k1) {
  if (a.causal && k0 > q1) return false;
  const int bs = a.L.bs, nq = a.L.nq;
  for (int qb = q0 / bs; qb <= q1 / bs; ++qb)
    for (int kb = k0 / bs; kb <= k1 / bs; ++kb)
      if (m[qb * nq + kb]) return true;
  return false;
}

__device__ __forceinline__ bool live(const AttnArgs& a, const uint8_t* m, int q, int k) {
  return m[(q / a.L.bs) * a.L.nq + (k / a.L.bs)] && (!a.causal || k <= q);
}

// Loads a [kKT, D] tile of rows [r0, r0+kKT) into smem as float, element (j, 2c+hf) holding
// column hf*D/2 + c so the two threads of a row read adjacent words.
template <typename T, int D>
__device__ __forceinline__ void load_tile(float (*dst)[D], const void* src, const int64_t* st3,
                                          int b, int h, int r0, int S) {
  constexpr int DH = D / 2;
  for (int i = threadIdx.x; i < kKT * D; i += blockDim.x) {
    const int j = i / D, col = i % D;
    const int r = r0 + j;
    float x = 0.f;
    if (r < S) x = ld<T>(src, b * st3[0] + h * st3[1] + (int64_t)r * st3[2] + col);
    dst[j][(col % DH) * 2 + col / DH] = x;
  }
}

template <typename T, int D>
__global__ void __launch_bounds__(128) simt_fwd_kernel(AttnArgs a) {
  constexpr int DH = D / 2;
  __shared__ float sK[kKT][D];
  __shared__ float sV[kKT][D];
  __shared__ float sMean[D];
  __shared__ int s_ok;
  if (threadIdx.x == 0) {
    s_ok = plan_matches(a);
    if (!s_ok) record_device_error(DEV_ERR_PLAN, 1);
  }
  __syncthreads();
  if (!s_ok) return;
  const int bh = blockIdx.y, b = bh / a.H, h = bh % a.H;
  if (!plan_unit_selected(a.plan, a.L, b, h)) return;   // a unit this plan does not compute
  const int q0 = blockIdx.x * kQT, q1 = min(q0 + kQT, a.S) - 1;
  const int r = threadIdx.x >> 1, hf = threadIdx.x & 1;
  const int row = q0 + r;
  const bool row_ok = row < a.S;
  const uint8_t* m = group_mask(a, b, h);

  float qv[DH], o[DH];
  const int64_t qoff = b * a.qs[0] + h * a.qs[1] + (int64_t)(row_ok ? row : 0) * a.qs[2] + hf * DH;
#pragma unroll
  for (int c = 0; c < DH; ++c) { qv[c] = row_ok ? ld<T>(a.q, qoff + c) * a.scale : 0.f; o[c] = 0.f; }
  float mrun = -INFINITY, l = 0.f;

  for (int k0 = 0; k0 < a.S; k0 += kKT) {
    const int k1 = min(k0 + kKT, a.S) - 1;
    if (a.causal && k0 > q1) break;
    if (!tile_live(a, m, q0, q1, k0, k1)) continue;
    __syncthreads();
    load_tile<T, D>(sK, a.k, a.ks, b, h, k0, a.S);
    load_tile<T, D>(sV, a.v, a.vs, b, h, k0, a.S);
    __syncthreads();
    float s[kKT];
    float tmax = -INFINITY;
#pragma unroll
    for (int j = 0; j < kKT; ++j) {
      float acc = 0.f;
#pragma unroll
      for (int c = 0; c < DH; ++c) acc = fmaf(qv[c], sK[j][2 * c + hf], acc);
      acc += __shfl_xor_sync(0xffffffffu, acc, 1);
      const int key = k0 + j;
      const bool on = row_ok && key <= k1 && live(a, m, row, key);
      s[j] = on ? acc : -INFINITY;
      tmax = fmaxf(tmax, s[j]);
    }
    const float mnew = fmaxf(mrun, tmax);
    if (mnew == -INFINITY) continue;
    const float alpha = expf(mrun - mnew);
    l *= alpha;
#pragma unroll
    for (int c = 0; c < DH; ++c) o[c] *= alpha;
#pragma unroll
    for (int j = 0; j < kKT; ++j) {
      const float p = expf(s[j] - mnew);
      l += p;
#pragma unroll
      for (int c = 0; c < DH; ++c) o[c] = fmaf(p, sV[j][2 * c + hf], o[c]);
    }
    mrun = mnew;
  }

  const bool empty = row_ok && l == 0.f;
  if (__syncthreads_or(empty)) {   // rare: some row has no live score -> mean of all V rows
    for (int c = threadIdx.x; c < D; c += blockDim.x) {
      float acc = 0.f;
      for (int j = 0; j < a.S; ++j) acc += ld<T>(a.v, b * a.vs[0] + h * a.vs[1] + (int64_t)j * a.vs[2] + c);
      sMean[c] = acc / (float)a.S;
    }
    __syncthreads();
  }
  if (!row_ok) return;
  const int64_t ooff = b * a.os[0] + h * a.os[1] + (int64_t)row * a.os[2] + hf * DH;
  const float inv = empty ? 0.f : 1.f / l;
#pragma unroll
  for (int c = 0; c < DH; ++c) st<T>(a.o, ooff + c, empty ? sMean[hf * DH + c] : o[c] * inv);
  if (hf == 0) a.lse[(int64_t)bh * a.S + row] = empty ? kMaskFill : mrun + logf(l);
}

// delta[b,h,s] = rowsum(dO * O); ucol[b,h,:] = (1/S) * sum of dO over fully masked rows.
template <typename T>
__global__ void __launch_bounds__(256) bwd_prep_kernel(AttnArgs a) {
  const int bh = blockIdx.x, b = bh / a.H, h = bh % a.H;
  if (!plan_unit_selected(a.plan, a.L, b, h)) return;   // a unit this plan does not compute
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nw = blockDim.x >> 5;
  for (int row = warp; row < a.S; row += nw) {
    const int64_t oo = b * a.os[0] + h * a.os[1] + (int64_t)row * a.os[2];
    float acc = 0.f;
    for (int c = lane; c < a.D; c += 32) acc += ld<T>(a.dout, oo + c) * ld<T>(a.o, oo + c);
    acc = warp_sum(acc);
    if (lane == 0) a.delta[(int64_t)bh * a.S + row] = acc;
  }
  const uint8_t* qe = reinterpret_cast<const uint8_t*>(a.plan + a.L.qempty_off) +
                      (int64_t)a.L.group_of(b, h) * a.L.nq;
  for (int c = threadIdx.x; c < a.D; c += blockDim.x) {
    float acc = 0.f;
    for (int qb = 0; qb < a.L.nq; ++qb) {
      if (!qe[qb]) continue;
      for (int row = qb * a.L.bs; row < (qb + 1) * a.L.bs; ++row)
        acc += ld<T>(a.dout, b * a.os[0] + h * a.os[1] + (int64_t)row * a.os[2] + c);
    }
    a.ucol[(int64_t)bh * a.D + c] = acc / (float)a.S;
  }
}

template <typename T, int D>
__global__ void __launch_bounds__(128) simt_dq_kernel(AttnArgs a) {
  constexpr int DH = D / 2;
  __shared__ float sK[kKT][D];
  __shared__ float sV[kKT][D];
  __shared__ int s_ok;
  if (threadIdx.x == 0) {
    s_ok = plan_matches(a);
    if (!s_ok) record_device_error(DEV_ERR_PLAN, 2);
  }
  __syncthreads();
  if (!s_ok) return;
  const int bh = blockIdx.y, b = bh / a.H, h = bh % a.H;
  if (!plan_unit_selected(a.plan, a.L, b, h)) return;   // a unit this plan does not compute
  const int q0 = blockIdx.x * kQT, q1 = min(q0 + kQT, a.S) - 1;
  const int r = threadIdx.x >> 1, hf = threadIdx.x & 1;
  const int row = q0 + r;
  const bool row_ok = row < a.S;
  const uint8_t* m = group_mask(a, b, h);
  const int64_t qoff = b * a.qs[0] + h * a.qs[1] + (int64_t)(row_ok ? row : 0) * a.qs[2] + hf * DH;
  const int64_t ooff = b * a.os[0] + h * a.os[1] + (int64_t)(row_ok ? row : 0) * a.os[2] + hf * DH;
  float qv[DH], gv[DH], dq[DH];
#pragma unroll
  for (int c = 0; c < DH; ++c) {
    qv[c] = row_ok ? ld<T>(a.q, qoff + c) : 0.f;
    gv[c] = row_ok ? ld<T>(a.dout, ooff + c) : 0.f;
    dq[c] = 0.f;
  }
  const float lse = row_ok ? a.lse[(int64_t)bh * a.S + row] : 0.f;
  const float dl = row_ok ? a.delta[(int64_t)bh * a.S + row] : 0.f;
  for (int k0 = 0; k0 < a.S; k0 += kKT) {
    const int k1 = min(k0 + kKT, a.S) - 1;
    if (a.causal && k0 > q1) break;
    if (!tile_live(a, m, q0, q1, k0, k1)) continue;
    __syncthreads();
    load_tile<T, D>(sK, a.k, a.ks, b, h, k0, a.S);
    load_tile<T, D>(sV, a.v, a.vs, b, h, k0, a.S);
    __syncthreads();
#pragma unroll 4
    for (int j = 0; j < kKT; ++j) {
      float sdot = 0.f, pdot = 0.f;
#pragma unroll
      for (int c = 0; c < DH; ++c) {
        sdot = fmaf(qv[c], sK[j][2 * c + hf], sdot);
        pdot = fmaf(gv[c], sV[j][2 * c + hf], pdot);
      }
      sdot += __shfl_xor_sync(0xffffffffu, sdot, 1);
      pdot += __shfl_xor_sync(0xffffffffu, pdot, 1);
      const int key = k0 + j;
      const bool on = row_ok && key <= k1 && live(a, m, row, key);
      const float p = on ? expf(sdot * a.scale - lse) : 0.f;
      const float ds = p * (pdot - dl);
#pragma unroll
      for (int c = 0; c < DH; ++c) dq[c] = fmaf(ds, sK[j][2 * c + hf], dq[c]);
    }
  }
  if (!row_ok) return;
#pragma unroll
  for (int c = 0; c < DH; ++c) st<T>(a.dq, ooff + c, dq[c] * a.scale);
}

template <typename T, int D>
__global__ void __launch_bounds__(128) simt_dkdv_kernel(AttnArgs a) {
  constexpr int DH = D / 2;
  __shared__ float sQ[kKT][D];
  __shared__ float sG[kKT][D];
  __shared__ float sL[kKT], sD[kKT];
  __shared__ int s_ok;
  if (threadIdx.x == 0) {
    s_ok = plan_matches(a);
    if (!s_ok) record_device_error(DEV_ERR_PLAN, 3);
  }
  __syncthreads();
  if (!s_ok) return;
  const int bh = blockIdx.y, b = bh / a.H, h = bh % a.H;
  if (!plan_unit_selected(a.plan, a.L, b, h)) return;   // a unit this plan does not compute
  const int k0 = blockIdx.x * kQT, k1 = min(k0 + kQT, a.S) - 1;
  const int r = threadIdx.x >> 1, hf = threadIdx.x & 1;
  const int key = k0 + r;
  const bool key_ok = key < a.S;
  const uint8_t* m = group_mask(a, b, h);
  const int64_t koff = b * a.ks[0] + h * a.ks[1] + (int64_t)(key_ok ? key : 0) * a.ks[2] + hf * DH;
  const int64_t voff = b * a.vs[0] + h * a.vs[1] + (int64_t)(key_ok ? key : 0) * a.vs[2] + hf * DH;
  float kv[DH], vv[DH], dk[DH], dv[DH];
#pragma unroll
  for (int c = 0; c < DH; ++c) {
    kv[c] = key_ok ? ld<T>(a.k, koff + c) : 0.f;
    vv[c] = key_ok ? ld<T>(a.v, voff + c) : 0.f;
    dk[c] = 0.f;
    dv[c] = 0.f;
  }
  const int qstart = a.causal ? (k0 / kKT) * kKT : 0;
  for (int q0 = qstart; q0 < a.S; q0 += kKT) {
    const int q1 = min(q0 + kKT, a.S) - 1;
    if (!tile_live(a, m, q0, q1, k0, k1)) continue;
    __syncthreads();
    load_tile<T, D>(sQ, a.q, a.qs, b, h, q0, a.S);
    load_tile<T, D>(sG, a.dout, a.os, b, h, q0, a.S);
    if (threadIdx.x < kKT) {
      const int qr = q0 + threadIdx.x;
      sL[threadIdx.x] = qr < a.S ? a.lse[(int64_t)bh * a.S + qr] : 0.f;
      sD[threadIdx.x] = qr < a.S ? a.delta[(int64_t)bh * a.S + qr] : 0.f;
    }
    __syncthreads();
#pragma unroll 4
    for (int i = 0; i < kKT; ++i) {
      float sdot = 0.f, pdot = 0.f;
#pragma unroll
      for (int c = 0; c < DH; ++c) {
        sdot = fmaf(kv[c], sQ[i][2 * c + hf], sdot);
        pdot = fmaf(vv[c], sG[i][2 * c + hf], pdot);
      }
      sdot += __shfl_xor_sync(0xffffffffu, sdot, 1);
      pdot += __shfl_xor_sync(0xffffffffu, pdot, 1);
      const int qr = q0 + i;
      const bool on = key_ok && qr <= q1 && live(a, m, qr, key);
      const float p = on ? expf(sdot * a.scale - sL[i]) : 0.f;
      const float ds = p * (pdot - sD[i]);
#pragma unroll
      for (int c = 0; c < DH; ++c) {
        dv[c] = fmaf(p, sG[i][2 * c + hf], dv[c]);
        dk[c] = fmaf(ds, sQ[i][2 * c + hf], dk[c]);
      }
    }
  }
  if (!key_ok) return;
  const int64_t goff = b * a.os[0] + h * a.os[1] + (int64_t)key * a.os[2] + hf * DH;
  const float* u = a.ucol + (int64_t)bh * a.D + hf * DH;
#pragma unroll
  for (int c = 0; c < DH; ++c) {
    st<T>(a.dk, goff + c, dk[c] * a.scale);
    st<T>(a.dv, goff + c, dv[c] + u[c]);
  }
}

template <typename T, int D>
int launch_fwd(const AttnArgs& a, cudaStream_t s) {
  dim3 grid((a.S + kQT - 1) / kQT, a.B * a.H);
  simt_fwd_kernel<T, D><<<grid, 128, 0, s>>>(a);
  return check_launch("simt_fwd_kernel");
}

template <typename T, int D>
int launch_bwd(const AttnArgs& a, cudaStream_t s) {
  int st_;
  bwd_prep_kernel<T><<<a.B * a.H, 256, 0, s>>>(a);
  if ((st_ = check_launch("bwd_prep_kernel"))) return st_;
  dim3 grid((a.S + kQT - 1) / kQT, a.B * a.H);
  simt_dq_kernel<T, D><<<grid, 128, 0, s>>>(a);
  if ((st_ = check_launch("simt_dq_kernel"))) return st_;
  simt_dkdv_kernel<T, D><<<grid, 128, 0, s>>>(a);
  return check_launch("simt_dkdv_kernel");
}

template <typename T>
int dispatch_fwd(const AttnArgs& a, cudaStream_t s) {
  switch (a.D) {
    case 16: return launch_fwd<T, 16>(a, s);
    case 32: return launch_fwd<T, 32>(a, s);
    case 64: return launch_fwd<T, 64>(a, s);
    case 128: return launch_fwd<T, 128>(a, s);
  }
  return set_error(XSAKE_EUNSUPPORTED, "head_dim %d not in {16, 32, 64, 128}", a.D);
}

template <typename T>
int dispatch_bwd(const AttnArgs& a, cudaStream_t s) {
  switch (a.D) {
    case 16: return launch_bwd<T, 16>(a, s);
    case 32: return launch_bwd<T, 32>(a, s);
    case 64: return launch_bwd<T, 64>(a, s);
    case 128: return launch_bwd<T, 128>(a, s);
  }
  return set_error(XSAKE_EUNSUPPORTED, "head_dim %d not in {16, 32, 64, 128}", a.D);
}

}  // namespace

int simt_attn_fwd(const AttnArgs& a, int dtype, cudaStream_t s) {
  return dtype == XSAKE_F32 ? dispatch_fwd<float>(a, s) : dispatch_fwd<__nv_bfloat16>(a, s);
}

int simt_attn_bwd(const AttnArgs& a, int dtype, cudaStream_t s) {
  return dtype == XSAKE_F32 ? dispatch_bwd<float>(a, s) : dispatch_bwd<__nv_bfloat16>(a, s);
}

}  // namespace xsake
