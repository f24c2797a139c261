// Block-mask plan compiler (replaces the reference's per-call _broadcast_mask and the token
// mask expansion, kernels/pallas/sparse_attention.py:76-81 and :286-298).
//
// Three small launches, all stream-ordered and deterministic:
//   plan_rows_kernel   copy the mask, mark fully masked q-blocks, count entries per row
//   plan_scan_kernel   (one CTA) prefix sums, header, plan statistics, work-item order
//   plan_fill_kernel   write the entries of every row in ascending chunk order
#include "common.cuh"
#include "plan.cuh"

XSAKE_DEFINE_DEVICE_ERROR(plan)

namespace xsake {

__device__ __forceinline__ bool mask_at(const uint8_t* m, const PlanLayout& L, int g, int qb, int kb) {
  return m[((int64_t)g * L.nq + qb) * L.nq + kb] != 0;
}

// Flags of kv chunk c for forward pair row (g, t); 0 when neither half attends it.
__device__ __forceinline__ int32_t fwd_flags(const uint8_t* m, const PlanLayout& L, int g, int t, int c) {
  int32_t f = 0;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int qc = 2 * t + h;
    if (qc >= L.n64) continue;
    if (L.causal && c > qc) continue;
    if (!mask_at(m, L, g, qc * 64 / L.bs, c * 64 / L.bs)) continue;
    f |= (h ? kFlagActive1 : kFlagActive0);
    if (L.causal && c == qc) f |= (h ? kFlagDiag1 : kFlagDiag0);
  }
  return f;
}

// Flags of q chunk c for backward kv-pair column (g, u); halves are kv chunks 2u, 2u+1.
__device__ __forceinline__ int32_t bwd_flags(const uint8_t* m, const PlanLayout& L, int g, int u, int c) {
  int32_t f = 0;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int kc = 2 * u + h;
    if (kc >= L.n64) continue;
    if (L.causal && kc > c) continue;
    if (!mask_at(m, L, g, c * 64 / L.bs, kc * 64 / L.bs)) continue;
    f |= (h ? kFlagActive1 : kFlagActive0);
    if (L.causal && c == kc) f |= (h ? kFlagDiag1 : kFlagDiag0);
  }
  return f;
}

__global__ void plan_rows_kernel(PlanLayout L, const uint8_t* __restrict__ mask, int32_t* __restrict__ plan) {
  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t nthreads = (int64_t)gridDim.x * blockDim.x;
  uint8_t* pmask = reinterpret_cast<uint8_t*>(plan + L.mask_off);
  const int64_t mask_bytes = (int64_t)L.Bm * L.Hm * L.nq * L.nq;
  for (int64_t i = tid; i < mask_bytes; i += nthreads) pmask[i] = mask[i] ? 1 : 0;

  uint8_t* qempty = reinterpret_cast<uint8_t*>(plan + L.qempty_off);
  const int64_t nqrows = (int64_t)L.Bm * L.Hm * L.nq;
  for (int64_t r = tid; r < nqrows; r += nthreads) {
    const int g = (int)(r / L.nq), i = (int)(r % L.nq);
    const int jmax = L.causal ? i : L.nq - 1;
    bool any = false;
    for (int j = 0; j <= jmax && !any; ++j) any = mask_at(mask, L, g, i, j);
    qempty[r] = any ? 0 : 1;
  }
  if (!L.has_csr) return;
  int32_t* frow = plan + L.f_rowptr_off;
  int32_t* brow = plan + L.b_rowptr_off;
  for (int64_t r = tid; r < L.nrows; r += nthreads) {
    const int g = (int)(r / L.npairs), t = (int)(r % L.npairs);
    int nf = 0, nb = 0;
    for (int c = 0; c < L.n64; ++c) {
      nf += fwd_flags(mask, L, g, t, c) != 0;
      nb += bwd_flags(mask, L, g, t, c) != 0;
    }
    frow[r + 1] = nf;
    brow[r + 1] = nb;
  }
}

// Warp-wide exclusive scan of rowptr[1..n] (counts) in place, rowptr[0] = 0.
__device__ int64_t warp_scan_rowptr(int32_t* rowptr, int n) {
  const int lane = threadIdx.x & 31;
  int32_t carry = 0;
  if (lane == 0) rowptr[0] = 0;
  for (int base = 0; base < n; base += 32) {
    const int r = base + lane;
    int32_t v = (r < n) ? rowptr[r + 1] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int32_t y = __shfl_up_sync(0xffffffffu, v, o);
      if (lane >= o) v += y;
    }
    if (r < n) rowptr[r + 1] = v + carry;
    carry += __shfl_sync(0xffffffffu, v, 31);
  }
  return carry;
}

// Stable order of work items by descending cost, by one warp (deterministic).
__device__ void order_items(const PlanLayout& L, const int32_t* rowptr, int32_t* items, int nitems,
                            int nper, int32_t* hist /* smem, n64 + 2 */) {
  const int lane = threadIdx.x & 31;
  const int nb = L.n64 + 1;
  for (int c = lane; c <= nb; c += 32) hist[c] = 0;
  __syncwarp();
  auto cost_of = [&](int i) {
    const int t = i % nper;
    const int bh = i / nper;
    const int g = L.group_of(bh / L.H, bh % L.H);
    const int r = g * nper + t;
    return rowptr[r + 1] - rowptr[r];
  };
  for (int base = 0; base < nitems; base += 32) {
    const int i = base + lane;
    const int c = (i < nitems) ? cost_of(i) : -1;
    const unsigned grp = __match_any_sync(0xffffffffu, c);
    const int leader = __ffs(grp) - 1;
    if (c >= 0 && lane == leader) hist[c] += __popc(grp);
    __syncwarp();
  }
  if (lane == 0) {  // bucket bases, largest cost first
    int32_t acc = 0;
    for (int c = nb - 1; c >= 0; --c) {
      const int32_t n = hist[c];
      hist[c] = acc;
      acc += n;
    }
  }
  __syncwarp();
  for (int base = 0; base < nitems; base += 32) {
    const int i = base + lane;
    const int c = (i < nitems) ? cost_of(i) : -1;
    const unsigned grp = __match_any_sync(0xffffffffu, c);
    const int leader = __ffs(grp) - 1;
    const int rank = __popc(grp & ((1u << lane) - 1u));
    if (c >= 0) items[hist[c] + rank] = i;
    __syncwarp();
    if (c >= 0 && lane == leader) hist[c] += __popc(grp);
    __syncwarp();
  }
}

__global__ void plan_scan_kernel(PlanLayout L, int32_t* __restrict__ plan) {
  extern __shared__ int32_t smem[];
  __shared__ unsigned long long s_active, s_empty;
  const uint8_t* m = reinterpret_cast<const uint8_t*>(plan + L.mask_off);
  const uint8_t* qempty = reinterpret_cast<const uint8_t*>(plan + L.qempty_off);
  if (threadIdx.x == 0) { s_active = 0; s_empty = 0; }
  __syncthreads();
  const int64_t mult_b = (L.Bm == 1) ? L.B : 1, mult_h = (L.Hm == 1) ? L.H : 1;
  unsigned long long act = 0, emp = 0;
  const int64_t mask_bytes = (int64_t)L.Bm * L.Hm * L.nq * L.nq;
  for (int64_t i = threadIdx.x; i < mask_bytes; i += blockDim.x) {
    const int kb = (int)(i % L.nq), qb = (int)((i / L.nq) % L.nq);
    if (m[i] && (!L.causal || kb <= qb)) ++act;
  }
  for (int64_t r = threadIdx.x; r < (int64_t)L.Bm * L.Hm * L.nq; r += blockDim.x) emp += qempty[r];
  atomicAdd(&s_active, act);
  atomicAdd(&s_empty, emp);
  const int warp = threadIdx.x >> 5;
  int64_t f_nnz = 0, b_nnz = 0;
  if (L.has_csr) {
    if (warp == 0) f_nnz = warp_scan_rowptr(plan + L.f_rowptr_off, L.nrows);
    if (warp == 1) b_nnz = warp_scan_rowptr(plan + L.b_rowptr_off, L.nrows);
    __syncthreads();
    if (warp == 0) order_items(L, plan + L.f_rowptr_off, plan + L.f_items_off, L.nitems, L.npairs, smem);
    if (warp == 1)
      order_items(L, plan + L.b_rowptr_off, plan + L.b_items_off, L.nitems, L.npairs, smem + (L.n64 + 2));
  }
  __syncthreads();
  if (threadIdx.x == 0 || threadIdx.x == 32) {
    int32_t* hdr = plan;
    if (threadIdx.x == 0) {
      hdr[H_VERSION] = kPlanVersion;
      hdr[H_B] = L.B; hdr[H_H] = L.H; hdr[H_S] = L.S; hdr[H_BM] = L.Bm; hdr[H_HM] = L.Hm;
      hdr[H_BS] = L.bs; hdr[H_CAUSAL] = L.causal; hdr[H_HAS_CSR] = L.has_csr;
      hdr[H_F_NNZ] = (int32_t)f_nnz;
      int64_t tiles = 0;
      if (L.has_csr) {
        const int32_t* rp = plan + L.f_rowptr_off;
        for (int i = 0; i < L.nitems; ++i) {
          const int t = i % L.npairs, bh = i / L.npairs;
          const int r = L.group_of(bh / L.H, bh % L.H) * L.npairs + t;
          tiles += 2 * (rp[r + 1] - rp[r]);   // each entry is a 128x64 tile = two 64x64 tiles
        }
      }
      const int64_t active = (int64_t)s_active * mult_b * mult_h;
      const int64_t empty = (int64_t)s_empty * mult_b * mult_h;
      hdr[H_ACTIVE_LO] = (int32_t)(active & 0xffffffff); hdr[H_ACTIVE_HI] = (int32_t)(active >> 32);
      hdr[H_TILES_LO] = (int32_t)(tiles & 0xffffffff);   hdr[H_TILES_HI] = (int32_t)(tiles >> 32);
      hdr[H_EMPTY_LO] = (int32_t)(empty & 0xffffffff);   hdr[H_EMPTY_HI] = (int32_t)(empty >> 32);
      hdr[H_ITEMS_LO] = L.has_csr ? L.nitems : 0;        hdr[H_ITEMS_HI] = 0;
      // Forward pairing: the same query chunk of two units that share the mask when there are
      // two such units and pairing query chunks 2t, 2t+1 would leave more than 12% of the 64-row
      // halves it computes masked out (measured crossover: 67-80% useful halves favour unit
      // pairing by 3-8%, 98.5% favours query-chunk pairing by 7%).
      const int64_t units = (int64_t)(L.Bm == 1 ? L.B : 1) * (L.Hm == 1 ? L.H : 1);
      hdr[H_FWD_PAIR] = (L.has_csr && units >= 2 && 100 * active < 88 * tiles) ? 1 : 0;
      __threadfence();
      hdr[H_MAGIC] = kPlanMagic;
    } else {
      plan[H_B_NNZ] = (int32_t)b_nnz;
    }
  }
}

__global__ void plan_fill_kernel(PlanLayout L, int32_t* __restrict__ plan) {
  const uint8_t* m = reinterpret_cast<const uint8_t*>(plan + L.mask_off);
  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t nthreads = (int64_t)gridDim.x * blockDim.x;
  const int32_t* frow = plan + L.f_rowptr_off;
  const int32_t* brow = plan + L.b_rowptr_off;
  int32_t* fent = plan + L.f_entries_off;
  int32_t* bent = plan + L.b_entries_off;
  for (int64_t r = tid; r < 2 * (int64_t)L.nrows; r += nthreads) {
    const bool fwd = r < L.nrows;
    const int64_t rr = fwd ? r : r - L.nrows;
    const int g = (int)(rr / L.npairs), t = (int)(rr % L.npairs);
    int32_t pos = fwd ? frow[rr] : brow[rr];
    int32_t* ent = fwd ? fent : bent;
    for (int c = 0; c < L.n64; ++c) {
      const int32_t f = fwd ? fwd_flags(m, L, g, t, c) : bwd_flags(m, L, g, t, c);
      if (f) ent[pos++] = c | f;
    }
  }
}

int plan_layout_from_dims(const XsakeMaskDims* d, PlanLayout* L) {
  XSAKE_REQUIRE(d != nullptr, XSAKE_EINVAL, "dims is NULL");
  XSAKE_REQUIRE(d->batch > 0 && d->heads > 0 && d->seq > 0 && d->block_size > 0, XSAKE_EINVAL,
                "batch, heads, seq and block_size must be positive");
  XSAKE_REQUIRE(d->seq % d->block_size == 0, XSAKE_EINVAL,
                "block_size %d must divide seq %d", d->block_size, d->seq);
  XSAKE_REQUIRE(d->mask_batch == 1 || d->mask_batch == d->batch, XSAKE_EINVAL,
                "mask batch dim %d must be 1 or batch %d", d->mask_batch, d->batch);
  XSAKE_REQUIRE(d->mask_heads == 1 || d->mask_heads == d->heads, XSAKE_EINVAL,
                "mask heads dim %d must be 1 or heads %d", d->mask_heads, d->heads);
  XSAKE_REQUIRE((int64_t)d->seq / 64 < (1 << 20), XSAKE_EUNSUPPORTED, "seq too long");
  XSAKE_REQUIRE((int64_t)d->batch * d->heads * ((d->seq / 64 + 2) / 2) < (1ll << 31),
                XSAKE_EUNSUPPORTED, "too many work items");
  if (!L->init(d->batch, d->heads, d->seq, d->mask_batch, d->mask_heads, d->block_size, d->causal))
    return set_error(XSAKE_EINVAL, "invalid mask dims");
  return XSAKE_OK;
}

}  // namespace xsake

using namespace xsake;

extern "C" int xsake_mask_plan_bytes(const XsakeMaskDims* dims, size_t* bytes) {
  clear_error();
  XSAKE_REQUIRE(bytes != nullptr, XSAKE_EINVAL, "bytes is NULL");
  PlanLayout L;
  int st = plan_layout_from_dims(dims, &L);
  if (st) return st;
  *bytes = (size_t)L.total_words * 4;
  return XSAKE_OK;
}

extern "C" int xsake_mask_compile(const XsakeMaskDims* dims, const uint8_t* mask_dev, void* plan_dev,
                                  size_t plan_bytes, void* stream) {
  clear_error();
  PlanLayout L;
  int st = plan_layout_from_dims(dims, &L);
  if (st) return st;
  XSAKE_REQUIRE(mask_dev && plan_dev, XSAKE_EINVAL, "mask and plan must be device pointers");
  XSAKE_REQUIRE(plan_bytes >= (size_t)L.total_words * 4, XSAKE_EINVAL,
                "plan buffer too small: %zu < %lld bytes", plan_bytes, (long long)L.total_words * 4);
  XSAKE_REQUIRE(((uintptr_t)plan_dev & 15) == 0, XSAKE_EINVAL, "plan must be 16-byte aligned");
  DeviceInfo di;
  if ((st = device_info(&di))) return st;
  cudaStream_t s = as_stream(stream);
  const int64_t work = std::max<int64_t>((int64_t)L.Bm * L.Hm * L.nq * L.nq, 3 * (int64_t)L.nrows);
  const int blocks = (int)std::min<int64_t>((work + 255) / 256, 4 * (int64_t)di.sm_count);
  plan_rows_kernel<<<std::max(blocks, 1), 256, 0, s>>>(L, mask_dev, (int32_t*)plan_dev);
  if ((st = check_launch("plan_rows_kernel"))) return st;
  const size_t smem = 2 * (size_t)(L.n64 + 2) * sizeof(int32_t);
  XSAKE_REQUIRE(smem <= 48 * 1024, XSAKE_EUNSUPPORTED, "seq too long for the plan compiler");
  plan_scan_kernel<<<1, 1024, smem, s>>>(L, (int32_t*)plan_dev);
  if ((st = check_launch("plan_scan_kernel"))) return st;
  if (L.has_csr) {
    const int fb = (int)std::min<int64_t>((3 * (int64_t)L.nrows + 127) / 128, 4 * (int64_t)di.sm_count);
    plan_fill_kernel<<<std::max(fb, 1), 128, 0, s>>>(L, (int32_t*)plan_dev);
    if ((st = check_launch("plan_fill_kernel"))) return st;
  }
  return XSAKE_OK;
}

extern "C" int xsake_mask_plan_stats(const void* plan_dev, void* stream, int64_t out[4]) {
  clear_error();
  XSAKE_REQUIRE(plan_dev && out, XSAKE_EINVAL, "NULL argument");
  int32_t hdr[kPlanHeaderWords];
  cudaStream_t s = as_stream(stream);
  XSAKE_CUDA_TRY(cudaMemcpyAsync(hdr, plan_dev, sizeof(hdr), cudaMemcpyDeviceToHost, s));
  XSAKE_CUDA_TRY(cudaStreamSynchronize(s));
  XSAKE_REQUIRE(hdr[H_MAGIC] == kPlanMagic, XSAKE_EINVAL, "not a compiled plan");
  auto u64 = [&](int lo) { return (int64_t)(uint32_t)hdr[lo] | ((int64_t)hdr[lo + 1] << 32); };
  out[0] = u64(H_ACTIVE_LO);
  out[1] = u64(H_TILES_LO);
  out[2] = u64(H_EMPTY_LO);
  out[3] = u64(H_ITEMS_LO);
  return XSAKE_OK;
}
