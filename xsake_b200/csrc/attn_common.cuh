// Arguments shared by the attention kernels and their host launchers.
#pragma once

#include <cuda.h>

#include "common.cuh"
#include "plan.cuh"

namespace xsake {

struct AttnArgs {
  const void* q;
  const void* k;
  const void* v;
  void* o;
  float* lse;
  const void* dout;
  void* dq;
  void* dk;
  void* dv;
  float* delta;      // [B*H*S] rowsum(dO * O)            (backward workspace)
  float* ucol;       // [B*H*D] (1/S) * sum of dO over fully masked rows (backward workspace)
  int64_t qs[3], ks[3], vs[3], os[3];
  int B, H, S, D;
  float scale;
  int causal;
  PlanLayout L;
  const int32_t* plan;
};

// Plan header check run by thread 0 of a kernel; false when the plan does not belong to
// this call (the caller then records DEV_ERR_PLAN and exits).
__device__ __forceinline__ bool plan_matches(const AttnArgs& a) {
  const int32_t* h = a.plan;
  return h[H_MAGIC] == kPlanMagic && h[H_VERSION] == kPlanVersion && h[H_B] == a.B &&
         h[H_H] == a.H && h[H_S] == a.S && h[H_BM] == a.L.Bm && h[H_HM] == a.L.Hm &&
         h[H_BS] == a.L.bs && h[H_CAUSAL] == a.L.causal;
}

// Launchers (return XSAKE_* codes).
int simt_attn_fwd(const AttnArgs& a, int dtype, cudaStream_t s);
int simt_attn_bwd(const AttnArgs& a, int dtype, cudaStream_t s);
int tc_attn_fwd(const AttnArgs& a, void* ws, size_t ws_bytes, cudaStream_t s);
size_t tc_attn_fwd_workspace();   // bytes the tensor-core forward needs
bool tc_attn_fwd_supported(const AttnArgs& a, int dtype);
int tc_attn_bwd(const AttnArgs& a, void* ws, size_t ws_bytes, cudaStream_t s);
bool tc_attn_bwd_supported(const AttnArgs& a, int dtype);

// Block mask of the entropy of masked weights (xsake_attn_entropy): the compiled plan (header
// checked on the device) and its mask copy [Bm, Hm, nq, nq].
struct EtMask {
  const int32_t* plan;
  const uint8_t* mask;
  int Bm, Hm, bs, causal;
};

// 4-D bf16 TMA map over [B, H, S, 64] with (b, h, s) element strides; box = rows x 64,
// SWIZZLE_128B.  Defined in attn_fwd_tc.cu.
int tc_make_map(CUtensorMap* map, const void* base, const int64_t st[3], int B, int H, int S, int rows);

}  // namespace xsake
