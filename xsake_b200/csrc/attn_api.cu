// C-ABI entry points of the attention path: argument validation and kernel selection.
//   bf16, head_dim 64, block_size % 64 == 0, 16-byte aligned rows -> tensor-core forward
//   everything else (fp32, other head dims or block sizes)       -> CUDA-core kernels
// The backward follows the same split: tensor-core kernels for bf16 / head_dim 64 / 64-multiple
// blocks with 16-byte aligned rows, CUDA-core kernels otherwise.
// Every kernel checks the plan header against the call (DEV_ERR_PLAN on mismatch).
#include "attn_common.cuh"

#include <algorithm>
#include <math.h>

namespace xsake {

int plan_layout_from_dims(const XsakeMaskDims* d, PlanLayout* L);

namespace {

int build_args(const XsakeAttnDesc* d, const void* plan, AttnArgs* a) {
  XSAKE_REQUIRE(d != nullptr, XSAKE_EINVAL, "desc is NULL");
  XSAKE_REQUIRE(plan != nullptr, XSAKE_EINVAL, "plan is NULL");
  XSAKE_REQUIRE(((uintptr_t)plan & 15) == 0, XSAKE_EINVAL, "plan must be 16-byte aligned");
  XSAKE_REQUIRE(d->dtype == XSAKE_F32 || d->dtype == XSAKE_BF16, XSAKE_EINVAL, "dtype %d", d->dtype);
  XSAKE_REQUIRE(d->batch > 0 && d->heads > 0 && d->seq > 0 && d->head_dim > 0, XSAKE_EINVAL,
                "batch, heads, seq, head_dim must be positive");
  const int64_t* sts[4] = {d->q_stride, d->k_stride, d->v_stride, d->o_stride};
  for (auto st : sts)
    for (int i = 0; i < 3; ++i) XSAKE_REQUIRE(st[i] > 0, XSAKE_EINVAL, "strides must be positive");
  *a = AttnArgs{};
  a->B = d->batch;
  a->H = d->heads;
  a->S = d->seq;
  a->D = d->head_dim;
  a->causal = d->causal ? 1 : 0;
  a->scale = d->scale > 0.f ? d->scale : 1.0f / sqrtf((float)d->head_dim);
  for (int i = 0; i < 3; ++i) {
    a->qs[i] = d->q_stride[i];
    a->ks[i] = d->k_stride[i];
    a->vs[i] = d->v_stride[i];
    a->os[i] = d->o_stride[i];
  }
  a->plan = reinterpret_cast<const int32_t*>(plan);
  XsakeMaskDims md{d->batch, d->heads, d->seq, d->mask_batch, d->mask_heads, d->block_size, d->causal};
  return plan_layout_from_dims(&md, &a->L);
}

}  // namespace
}  // namespace xsake

using namespace xsake;

extern "C" int xsake_attn_fwd_workspace_size(const XsakeAttnDesc* desc, size_t* bytes) {
  clear_error();
  XSAKE_REQUIRE(desc && bytes, XSAKE_EINVAL, "NULL argument");
  // Work-item counter and split-piece partials of the persistent tensor-core kernel; the
  // CUDA-core kernels need none.
  const bool tc = desc->dtype == XSAKE_BF16 && desc->head_dim == 64 && desc->block_size > 0 &&
                  desc->block_size % 64 == 0 && desc->seq % 64 == 0;
  *bytes = tc ? tc_attn_fwd_workspace() : 256;
  return XSAKE_OK;
}

extern "C" int xsake_attn_fwd(const XsakeAttnDesc* desc, const void* plan_dev, const void* q_dev,
                              const void* k_dev, const void* v_dev, void* o_dev, float* lse_dev,
                              void* workspace_dev, size_t workspace_bytes, void* stream) {
  clear_error();
  AttnArgs a;
  int st = build_args(desc, plan_dev, &a);
  if (st) return st;
  XSAKE_REQUIRE(q_dev && k_dev && v_dev && o_dev && lse_dev, XSAKE_EINVAL, "NULL tensor pointer");
  a.q = q_dev;
  a.k = k_dev;
  a.v = v_dev;
  a.o = o_dev;
  a.lse = lse_dev;
  cudaStream_t s = as_stream(stream);
  if (tc_attn_fwd_supported(a, desc->dtype)) return tc_attn_fwd(a, workspace_dev, workspace_bytes, s);
  return simt_attn_fwd(a, desc->dtype, s);
}

extern "C" int xsake_attn_bwd_workspace_size(const XsakeAttnDesc* desc, size_t* bytes) {
  clear_error();
  XSAKE_REQUIRE(desc && bytes, XSAKE_EINVAL, "NULL argument");
  const int64_t bh = (int64_t)desc->batch * desc->heads;
  // delta [B*H*S] | ucol [B*H*D] | -lse*log2e [B*H*S] | work-item counters | 32 bytes per query
  // row of bias operands (tensor-core backward); the CUDA-core backward uses the first two sections.
  const size_t rows = align_up((size_t)(bh * desc->seq) * 4, 256);
  *bytes = 2 * rows + align_up((size_t)(bh * desc->head_dim) * 4, 256) + 256 + (size_t)(bh * desc->seq) * 32;
  return XSAKE_OK;
}

extern "C" int xsake_attn_bwd(const XsakeAttnDesc* desc, const void* plan_dev, const void* q_dev,
                              const void* k_dev, const void* v_dev, const void* o_dev,
                              const float* lse_dev, const void* do_dev, void* dq_dev, void* dk_dev,
                              void* dv_dev, void* workspace_dev, size_t workspace_bytes, void* stream) {
  clear_error();
  AttnArgs a;
  int st = build_args(desc, plan_dev, &a);
  if (st) return st;
  XSAKE_REQUIRE(q_dev && k_dev && v_dev && o_dev && lse_dev && do_dev && dq_dev && dk_dev && dv_dev,
                XSAKE_EINVAL, "NULL tensor pointer");
  size_t need = 0;
  xsake_attn_bwd_workspace_size(desc, &need);
  XSAKE_REQUIRE(workspace_dev != nullptr && workspace_bytes >= need, XSAKE_EINVAL,
                "workspace too small: %zu < %zu bytes", workspace_bytes, need);
  a.q = q_dev;
  a.k = k_dev;
  a.v = v_dev;
  a.o = const_cast<void*>(o_dev);
  a.lse = const_cast<float*>(lse_dev);
  a.dout = do_dev;
  a.dq = dq_dev;
  a.dk = dk_dev;
  a.dv = dv_dev;
  XSAKE_REQUIRE(((uintptr_t)workspace_dev & 255) == 0, XSAKE_EINVAL, "workspace must be 256-byte aligned");
  cudaStream_t s = as_stream(stream);
  if (tc_attn_bwd_supported(a, desc->dtype)) return tc_attn_bwd(a, workspace_dev, workspace_bytes, s);
  const int64_t bh = (int64_t)a.B * a.H;
  a.delta = reinterpret_cast<float*>(workspace_dev);
  a.ucol = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(workspace_dev) + align_up((size_t)(bh * a.S) * 4, 256));
  return simt_attn_bwd(a, desc->dtype, s);
}
