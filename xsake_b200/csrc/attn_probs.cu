// Dense attention probabilities and fused QK -> entropy, in fp32 on the CUDA cores.
//
//   probs    the second output of sparse_attention_reference (kernels/pallas/sparse_attention.py:
//            45-91): P = softmax over all S keys of the scaled scores with masked entries set to
//            finfo(float32).min (:87), token mask = block mask expanded (:76-77) and, if causal,
//            cut to keys <= query (:79-81).  A fully masked row therefore gets 1/S everywhere.
//            The reference's calibration (training/trainer.py:79-117) collects these weights.
//   entropy  compute_attention_entropy (kernels/hads/hads_pattern.py:36-50) of softmax(Q K^T *
//            scale) without materialising P: per row H = -sum_k c log c, c = clip(p, 1e-9, 1),
//            summed per head in fp64 in a fixed order (per-CTA partials, then one pass per head).
//   masked entropy  the same of the masked weights `probs` gives (the weights the reference's
//            calibration collects from layer 0, training/trainer.py:79-117): masked keys have
//            p = 0 and so contribute the clipped 1e-9 term, as in the reference.
//
// Scores are fp32 products (TF32 would move entropies by ~1e-3).  CTA = 256 threads on a tile of
// 64 query rows of one (b, h); K arrives in 64-key tiles staged transposed in shared memory;
// each thread owns a 4x4 block of the 64x64 score tile.  Two passes over the keys: row max and
// sum (online), then the probabilities (written, or turned into entropy terms).
#include "attn_common.cuh"

#include <algorithm>

XSAKE_DEFINE_DEVICE_ERROR(probs)

namespace xsake {
namespace {

constexpr int kRows = 64, kKeys = 64, kThreadsP = 256;
constexpr float kClipLo = 1e-9f;

struct ProbsArgs {
  const void* q;
  const void* k;
  int64_t qs[3], ks[3];
  int B, H, S;
  float scale;
  int causal;
  const int32_t* plan;        // probs: compiled plan (header checked, mask copy used)
  const uint8_t* mask;        // plan's mask copy [Bm, Hm, nq, nq] or NULL (no block mask)
  int Bm, Hm, bs;
  float* p;                   // probs: [B, H, S, S] fp32
  double* partial;            // entropy: [B * H * S / 64] per-CTA sums
};

template <typename T, int D>
__device__ __forceinline__ void stage_transposed(float (*dst)[kRows + 4], const T* src, const int64_t* st, int b,
                                                 int h, int r0, int S) {
  // dst[d][r] = src[b, h, r0 + r, d]; rows past S are zero.
  for (int i = threadIdx.x; i < kRows * D; i += kThreadsP) {
    const int r = i / D, d = i % D;
    const int row = r0 + r;
    dst[d][r] = row < S ? DT<T>::to_f(src[b * st[0] + h * st[1] + (int64_t)row * st[2] + d]) : 0.f;
  }
}

// exp(x - mn) scaled sum update that stays 0 (not NaN) while no finite score has been seen
__device__ __forceinline__ float rescale_sum(float l, float m, float mn) {
  return (m == -INFINITY) ? 0.f : l * __expf(m - mn);
}

// MODE: kEntropy (no mask), kProbs (masked weights), kMaskedEntropy (entropy of the masked weights)
constexpr int kEntropy = 0, kProbs = 1, kMaskedEntropy = 2;

template <typename T, int D, int MODE>
__global__ void __launch_bounds__(kThreadsP) probs_kernel(ProbsArgs a) {
  constexpr bool PROBS = MODE == kProbs;
  constexpr bool MASKED = MODE != kEntropy;
  __shared__ float sQ[D][kRows + 4];
  __shared__ float sK[D][kKeys + 4];
  __shared__ double sRow[kRows];
  __shared__ int s_ok;
  if (MASKED) {
    if (threadIdx.x == 0) {
      const int32_t* hd = a.plan;
      s_ok = hd[H_MAGIC] == kPlanMagic && hd[H_VERSION] == kPlanVersion && hd[H_B] == a.B && hd[H_H] == a.H &&
             hd[H_S] == a.S && hd[H_BM] == a.Bm && hd[H_HM] == a.Hm && hd[H_BS] == a.bs && hd[H_CAUSAL] == a.causal;
      if (!s_ok) record_device_error(DEV_ERR_PLAN, 40);
    }
    __syncthreads();
    if (!s_ok) return;
  }
  const int bh = blockIdx.y, b = bh / a.H, h = bh % a.H;
  const int q0 = blockIdx.x * kRows;
  const int t = threadIdx.x, ti = (t >> 4) * 4, tj = (t & 15) * 4;   // 4 rows x 4 keys
  const T* q = reinterpret_cast<const T*>(a.q);
  const T* k = reinterpret_cast<const T*>(a.k);
  stage_transposed<T, D>(sQ, q, a.qs, b, h, q0, a.S);
  const uint8_t* mrow = nullptr;
  int nq = 0;
  if (MASKED && a.mask) {
    nq = a.S / a.bs;
    mrow = a.mask + (int64_t)((a.Bm == 1 ? 0 : b) * a.Hm + (a.Hm == 1 ? 0 : h)) * nq * nq;
  }
  float m[4], l[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) { m[i] = -INFINITY; l[i] = 0.f; }

  // scores of this thread's 4x4 block for the K tile at k0 (masked entries -> finfo.min)
  auto scores = [&](int k0, float (&s)[4][4]) {
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) s[i][j] = 0.f;
#pragma unroll 8
    for (int d = 0; d < D; ++d) {
      const float4 qv = *reinterpret_cast<const float4*>(&sQ[d][ti]);
      const float4 kv = *reinterpret_cast<const float4*>(&sK[d][tj]);
      const float qa[4] = {qv.x, qv.y, qv.z, qv.w}, ka[4] = {kv.x, kv.y, kv.z, kv.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) s[i][j] = fmaf(qa[i], ka[j], s[i][j]);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int row = q0 + ti + i;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int key = k0 + tj + j;
        float v = s[i][j] * a.scale;
        if (key >= a.S) v = -INFINITY;                      // outside the sequence: no weight
        else if (MASKED) {
          bool keep = !a.causal || key <= row;
          if (keep && mrow) keep = mrow[(int64_t)(min(row, a.S - 1) / a.bs) * nq + key / a.bs] != 0;
          if (!keep) v = kMaskFill;
        }
        s[i][j] = v;
      }
    }
  };

  // ---- pass 1: row max and sum
  for (int k0 = 0; k0 < a.S; k0 += kKeys) {
    __syncthreads();
    stage_transposed<T, D>(sK, k, a.ks, b, h, k0, a.S);
    __syncthreads();
    float s[4][4];
    scores(k0, s);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float mx = fmaxf(fmaxf(s[i][0], s[i][1]), fmaxf(s[i][2], s[i][3]));
      const float mn = fmaxf(m[i], mx);
      if (mn == -INFINITY) continue;                       // only keys past the end so far
      float acc = rescale_sum(l[i], m[i], mn);
#pragma unroll
      for (int j = 0; j < 4; ++j) acc += __expf(s[i][j] - mn);
      m[i] = mn;
      l[i] = acc;
    }
  }
  // combine over the 16 threads that share these rows (lanes t, t^1, .., t^8 of a half-warp)
#pragma unroll
  for (int i = 0; i < 4; ++i) {
#pragma unroll
    for (int o = 1; o < 16; o <<= 1) {
      const float mo = __shfl_xor_sync(0xffffffffu, m[i], o), lo = __shfl_xor_sync(0xffffffffu, l[i], o);
      const float mn = fmaxf(m[i], mo);
      l[i] = rescale_sum(l[i], m[i], mn) + rescale_sum(lo, mo, mn);
      m[i] = mn;
    }
  }
  float inv[4], ent[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) { inv[i] = 1.f / l[i]; ent[i] = 0.f; }

  // ---- pass 2: probabilities
  for (int k0 = 0; k0 < a.S; k0 += kKeys) {
    __syncthreads();
    stage_transposed<T, D>(sK, k, a.ks, b, h, k0, a.S);
    __syncthreads();
    float s[4][4];
    scores(k0, s);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float pr[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) pr[j] = __expf(s[i][j] - m[i]) * inv[i];
      const int row = q0 + ti + i;
      if (PROBS) {
        if (row < a.S) {
          float* dst = a.p + ((int64_t)bh * a.S + row) * a.S + k0 + tj;
          if (k0 + tj + 3 < a.S && ((a.S & 3) == 0)) {
            *reinterpret_cast<float4*>(dst) = make_float4(pr[0], pr[1], pr[2], pr[3]);
          } else {
#pragma unroll
            for (int j = 0; j < 4; ++j)
              if (k0 + tj + j < a.S) dst[j] = pr[j];
          }
        }
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          if (k0 + tj + j < a.S) {
            const float c = fminf(fmaxf(pr[j], kClipLo), 1.0f);
            ent[i] = fmaf(c, __logf(c), ent[i]);
          }
        }
      }
    }
  }
  if (!PROBS) {
    // per-row entropy: sum over the 16 threads of the row, then the CTA's rows in a fixed order
#pragma unroll
    for (int i = 0; i < 4; ++i) {
#pragma unroll
      for (int o = 1; o < 16; o <<= 1) ent[i] += __shfl_xor_sync(0xffffffffu, ent[i], o);
    }
    if ((t & 15) == 0) {
#pragma unroll
      for (int i = 0; i < 4; ++i) sRow[ti + i] = (q0 + ti + i < a.S) ? -(double)ent[i] : 0.0;
    }
    __syncthreads();
    if (t == 0) {
      double acc = 0.0;
      for (int r = 0; r < kRows; ++r) acc += sRow[r];
      a.partial[(int64_t)bh * gridDim.x + blockIdx.x] = acc;
    }
  }
}

// One CTA per head: thread t sums partials t, t + 256, ... (in (b, tile) order), then a fixed
// shared-memory tree; the order depends only on the shapes.
__global__ void __launch_bounds__(256) probs_heads_kernel(const double* __restrict__ partial, int B, int H,
                                                          int per_bh, double* __restrict__ head_sums) {
  __shared__ double red[256];
  const int h = blockIdx.x;
  const int64_t n = (int64_t)B * per_bh;
  double acc = 0.0;
  for (int64_t i = threadIdx.x; i < n; i += 256) {
    const int64_t b = i / per_bh, c = i - b * per_bh;
    acc += partial[(b * H + h) * per_bh + c];
  }
  red[threadIdx.x] = acc;
  __syncthreads();
  for (int w = 128; w > 0; w >>= 1) {
    if ((int)threadIdx.x < w) red[threadIdx.x] += red[threadIdx.x + w];
    __syncthreads();
  }
  if (threadIdx.x == 0) head_sums[h] = red[0];
}

template <typename T, int MODE>
int launch(const ProbsArgs& a, int D, cudaStream_t s) {
  dim3 grid((a.S + kRows - 1) / kRows, a.B * a.H);
  switch (D) {
    case 32: probs_kernel<T, 32, MODE><<<grid, kThreadsP, 0, s>>>(a); break;
    case 64: probs_kernel<T, 64, MODE><<<grid, kThreadsP, 0, s>>>(a); break;
    default: return set_error(XSAKE_EUNSUPPORTED, "head_dim %d not in {32, 64}", D);
  }
  return check_launch(MODE == kProbs ? "probs_kernel" : "entropy_qk_kernel");
}

}  // namespace

int plan_layout_from_dims(const XsakeMaskDims* d, PlanLayout* L);
size_t entropy_tc_split_bytes(int64_t batch, int64_t heads, int64_t seq);
int entropy_tc(int dtype, const void* q, const void* k, const int64_t qs[3], const int64_t ks[3], int B, int H,
               int S, float scale, double* partial, void* split_buf, cudaStream_t s, const EtMask* mask,
               float* p_out);

}  // namespace xsake

using namespace xsake;

namespace xsake {
namespace {

// Arguments of the masked modes from an attention descriptor and a compiled plan.
int masked_args(const XsakeAttnDesc* desc, const void* plan_dev, const void* q_dev, const void* k_dev, ProbsArgs* out) {
  XSAKE_REQUIRE(desc && plan_dev && q_dev && k_dev, XSAKE_EINVAL, "NULL argument");
  XSAKE_REQUIRE(desc->dtype == XSAKE_F32 || desc->dtype == XSAKE_BF16, XSAKE_EINVAL, "dtype %d", desc->dtype);
  XSAKE_REQUIRE(desc->batch > 0 && desc->heads > 0 && desc->seq > 0, XSAKE_EINVAL, "dims must be positive");
  XsakeMaskDims md{desc->batch, desc->heads, desc->seq, desc->mask_batch, desc->mask_heads, desc->block_size,
                   desc->causal};
  PlanLayout L;
  int st = plan_layout_from_dims(&md, &L);
  if (st) return st;
  XSAKE_REQUIRE(((uintptr_t)plan_dev & 15) == 0, XSAKE_EINVAL, "plan must be 16-byte aligned");
  XSAKE_REQUIRE((int64_t)desc->batch * desc->heads < 65536, XSAKE_EUNSUPPORTED, "too many (batch, head) slices");
  ProbsArgs a{};
  a.q = q_dev;
  a.k = k_dev;
  for (int i = 0; i < 3; ++i) {
    a.qs[i] = desc->q_stride[i];
    a.ks[i] = desc->k_stride[i];
  }
  a.B = desc->batch;
  a.H = desc->heads;
  a.S = desc->seq;
  a.scale = desc->scale > 0.f ? desc->scale : 1.0f / sqrtf((float)desc->head_dim);
  a.causal = desc->causal ? 1 : 0;
  a.plan = reinterpret_cast<const int32_t*>(plan_dev);
  a.mask = reinterpret_cast<const uint8_t*>(a.plan + L.mask_off);
  a.Bm = L.Bm;
  a.Hm = L.Hm;
  a.bs = L.bs;
  *out = a;
  return XSAKE_OK;
}

}  // namespace
}  // namespace xsake

namespace xsake {
namespace {
// Rows the tensor-core kernel reads with 16-byte loads / TMA: base and (b, h, s) strides aligned.
bool tc_rows_aligned(int dtype, const void* q, const void* k, const int64_t qs[3], const int64_t ks[3]) {
  const int64_t al = dtype == XSAKE_F32 ? 4 : 8;
  bool ok = ((uintptr_t)q & 15) == 0 && ((uintptr_t)k & 15) == 0;
  for (int i = 0; i < 3; ++i) ok = ok && qs[i] % al == 0 && ks[i] % al == 0;
  return ok;
}

// Workspace: per-(b, h, 64-row tile) fp64 partials, then (from a 256-byte boundary) the bf16
// parts of K the tensor-core kernel reads for fp32 inputs.
size_t partial_bytes(int64_t batch, int64_t heads, int64_t seq) {
  return (size_t)(batch * heads * ((seq + kRows - 1) / kRows)) * sizeof(double);
}
size_t split_offset(int64_t batch, int64_t heads, int64_t seq) {
  return (partial_bytes(batch, heads, seq) + 255) / 256 * 256;
}
}  // namespace
}  // namespace xsake

extern "C" int xsake_attn_entropy(const XsakeAttnDesc* desc, const void* plan_dev, const void* q_dev,
                                  const void* k_dev, double* head_sums_dev, void* workspace_dev,
                                  size_t workspace_bytes, void* stream) {
  clear_error();
  ProbsArgs a;
  int st = masked_args(desc, plan_dev, q_dev, k_dev, &a);
  if (st) return st;
  XSAKE_REQUIRE(head_sums_dev != nullptr, XSAKE_EINVAL, "NULL argument");
  size_t need = 0;
  xsake_entropy_qk_workspace_size(a.B, a.H, a.S, &need);
  XSAKE_REQUIRE(workspace_dev && workspace_bytes >= need && ((uintptr_t)workspace_dev & 255) == 0, XSAKE_EINVAL,
                "workspace must be %zu bytes, 256-byte aligned (got %zu bytes)", need, workspace_bytes);
  a.partial = reinterpret_cast<double*>(workspace_dev);
  cudaStream_t s = as_stream(stream);
  int r;
  if (desc->head_dim == 64 && tc_rows_aligned(desc->dtype, q_dev, k_dev, a.qs, a.ks)) {
    const EtMask mk{a.plan, a.mask, a.Bm, a.Hm, a.bs, a.causal};
    void* split = reinterpret_cast<uint8_t*>(workspace_dev) + split_offset(a.B, a.H, a.S);
    r = entropy_tc(desc->dtype, q_dev, k_dev, a.qs, a.ks, a.B, a.H, a.S, a.scale, a.partial, split, s, &mk, nullptr);
  } else {
    r = desc->dtype == XSAKE_F32 ? launch<float, kMaskedEntropy>(a, desc->head_dim, s)
                                 : launch<__nv_bfloat16, kMaskedEntropy>(a, desc->head_dim, s);
  }
  if (r) return r;
  probs_heads_kernel<<<(unsigned)a.H, 256, 0, s>>>(a.partial, a.B, a.H, (a.S + kRows - 1) / kRows, head_sums_dev);
  return check_launch("probs_heads_kernel");
}

namespace xsake {
namespace {
// xsake_attn_probs(_ex): tensor cores at head_dim 64 when the inputs are bf16 or a workspace for
// the bf16 parts of fp32 K is given, CUDA cores otherwise.
int probs_impl(const XsakeAttnDesc* desc, const void* plan_dev, const void* q_dev, const void* k_dev, float* p_dev,
               void* ws, size_t ws_bytes, void* stream) {
  XSAKE_REQUIRE(p_dev != nullptr, XSAKE_EINVAL, "NULL argument");
  ProbsArgs a;
  int st = masked_args(desc, plan_dev, q_dev, k_dev, &a);
  if (st) return st;
  XSAKE_REQUIRE(((uintptr_t)p_dev & 15) == 0, XSAKE_EINVAL, "p must be 16-byte aligned");
  a.p = p_dev;
  cudaStream_t s = as_stream(stream);
  const bool f32 = desc->dtype == XSAKE_F32;
  const size_t split = f32 ? entropy_tc_split_bytes(a.B, a.H, a.S) : 0;
  const bool have_ws = !f32 || (ws && ws_bytes >= split && ((uintptr_t)ws & 255) == 0);
  if (desc->head_dim == 64 && have_ws && tc_rows_aligned(desc->dtype, q_dev, k_dev, a.qs, a.ks)) {
    const EtMask mk{a.plan, a.mask, a.Bm, a.Hm, a.bs, a.causal};
    return entropy_tc(desc->dtype, q_dev, k_dev, a.qs, a.ks, a.B, a.H, a.S, a.scale, nullptr, f32 ? ws : nullptr, s,
                      &mk, p_dev);
  }
  return f32 ? launch<float, kProbs>(a, desc->head_dim, s) : launch<__nv_bfloat16, kProbs>(a, desc->head_dim, s);
}
}  // namespace
}  // namespace xsake

extern "C" int xsake_attn_probs(const XsakeAttnDesc* desc, const void* plan_dev, const void* q_dev,
                                const void* k_dev, float* p_dev, void* stream) {
  clear_error();
  return probs_impl(desc, plan_dev, q_dev, k_dev, p_dev, nullptr, 0, stream);
}

extern "C" int xsake_attn_probs_workspace_size(const XsakeAttnDesc* desc, size_t* bytes) {
  clear_error();
  XSAKE_REQUIRE(desc && bytes && desc->batch > 0 && desc->heads > 0 && desc->seq > 0, XSAKE_EINVAL, "bad arguments");
  *bytes = std::max<size_t>(256, entropy_tc_split_bytes(desc->batch, desc->heads, desc->seq));
  return XSAKE_OK;
}

extern "C" int xsake_attn_probs_ex(const XsakeAttnDesc* desc, const void* plan_dev, const void* q_dev,
                                   const void* k_dev, float* p_dev, void* workspace_dev, size_t workspace_bytes,
                                   void* stream) {
  clear_error();
  XSAKE_REQUIRE(desc != nullptr, XSAKE_EINVAL, "NULL argument");
  size_t need = 0;
  int st = xsake_attn_probs_workspace_size(desc, &need);
  if (st) return st;
  XSAKE_REQUIRE(workspace_dev && workspace_bytes >= need && ((uintptr_t)workspace_dev & 255) == 0, XSAKE_EINVAL,
                "workspace must be %zu bytes, 256-byte aligned (got %zu bytes)", need, workspace_bytes);
  return probs_impl(desc, plan_dev, q_dev, k_dev, p_dev, workspace_dev, workspace_bytes, stream);
}

extern "C" int xsake_entropy_qk_workspace_size(int64_t batch, int64_t heads, int64_t seq, size_t* bytes) {
  clear_error();
  XSAKE_REQUIRE(bytes && batch > 0 && heads > 0 && seq > 0, XSAKE_EINVAL, "bad arguments");
  *bytes = split_offset(batch, heads, seq) + entropy_tc_split_bytes(batch, heads, seq);
  return XSAKE_OK;
}

extern "C" int xsake_entropy_qk(int32_t dtype, const void* q_dev, const void* k_dev, int64_t batch, int64_t heads,
                                int64_t seq, int64_t head_dim, float scale, double* head_sums_dev,
                                void* workspace_dev, size_t workspace_bytes, void* stream) {
  clear_error();
  XSAKE_REQUIRE(q_dev && k_dev && head_sums_dev, XSAKE_EINVAL, "NULL argument");
  XSAKE_REQUIRE(dtype == XSAKE_F32 || dtype == XSAKE_BF16, XSAKE_EINVAL, "dtype %d", dtype);
  XSAKE_REQUIRE(batch > 0 && heads > 0 && seq > 0 && head_dim > 0, XSAKE_EINVAL, "dims must be positive");
  XSAKE_REQUIRE(batch * heads < 65536 && seq < (1 << 30), XSAKE_EUNSUPPORTED, "too many (batch, head) slices");
  size_t need = 0;
  xsake_entropy_qk_workspace_size(batch, heads, seq, &need);
  XSAKE_REQUIRE(workspace_dev && workspace_bytes >= need && ((uintptr_t)workspace_dev & 255) == 0, XSAKE_EINVAL,
                "workspace must be %zu bytes, 256-byte aligned (got %zu bytes)", need, workspace_bytes);
  ProbsArgs a{};
  a.q = q_dev;
  a.k = k_dev;
  const int64_t st[3] = {heads * seq * head_dim, seq * head_dim, head_dim};
  for (int i = 0; i < 3; ++i) a.qs[i] = a.ks[i] = st[i];
  a.B = (int)batch;
  a.H = (int)heads;
  a.S = (int)seq;
  a.scale = scale > 0.f ? scale : 1.0f / sqrtf((float)head_dim);
  a.partial = reinterpret_cast<double*>(workspace_dev);
  cudaStream_t s = as_stream(stream);
  int r;
  if (head_dim == 64) {
    // tensor cores (three bf16 parts per fp32 operand, see entropy_tc.cu)
    void* split = reinterpret_cast<uint8_t*>(workspace_dev) + split_offset(batch, heads, seq);
    r = entropy_tc(dtype, q_dev, k_dev, st, st, a.B, a.H, a.S, a.scale, a.partial, split, s, nullptr, nullptr);
  } else {
    r = dtype == XSAKE_F32 ? launch<float, kEntropy>(a, (int)head_dim, s)
                           : launch<__nv_bfloat16, kEntropy>(a, (int)head_dim, s);
  }
  if (r) return r;
  probs_heads_kernel<<<(unsigned)heads, 256, 0, s>>>(a.partial, a.B, a.H, (a.S + kRows - 1) / kRows,
                                                     head_sums_dev);
  return check_launch("probs_heads_kernel");
}
