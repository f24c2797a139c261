// Block-mask plan compiler (replaces the reference's per-call _broadcast_mask and the token
// mask expansion, kernels/pallas/sparse_attention.py:76-81 and :286-298).
//
// Four small launches, all stream-ordered and deterministic:
//   plan_rows_kernel   copy the mask, mark fully masked q-blocks, count active blocks per
//                      q-block row, count entries per pair row and steps per query chunk
//   plan_scan_kernel   (one CTA) prefix sums of the entry counts, the unit selection
//   plan_fill_kernel   write the entries of every row in ascending chunk order
//   plan_work_kernel   (one CTA) selected-unit lists, statistics, backward item order, the
//                      forward pairing and the forward work table (with split pieces)
#include "common.cuh"
#include "plan.cuh"

#include <algorithm>

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

// Unit (b, h) that is member k of mask group g (members in ascending unit id).
__device__ __forceinline__ int unit_in_group(const PlanLayout& L, int g, int k) {
  const int fh = L.Hm == 1 ? L.H : 1;
  const int gb = L.Bm == 1 ? 0 : g / L.Hm, gh = L.Hm == 1 ? 0 : g % L.Hm;
  const int b = L.Bm == 1 ? k / fh : gb;
  const int h = L.Hm == 1 ? k % fh : gh;
  return b * L.H + h;
}

__global__ void plan_rows_kernel(PlanLayout L, const uint8_t* __restrict__ mask, const int32_t* __restrict__ units,
                                 int32_t* __restrict__ plan) {
  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t nthreads = (int64_t)gridDim.x * blockDim.x;
  uint8_t* pmask = reinterpret_cast<uint8_t*>(plan + L.mask_off);
  const int64_t mask_bytes = (int64_t)L.ngroups * L.nq * L.nq;
  for (int64_t i = tid; i < mask_bytes; i += nthreads) pmask[i] = mask[i] ? 1 : 0;

  // Selection: every unit without a list; else cleared here and set by plan_scan_kernel.
  uint8_t* usel = reinterpret_cast<uint8_t*>(plan + L.usel_off);
  for (int64_t u = tid; u < (int64_t)L.B * L.H; u += nthreads) usel[u] = units ? 0 : 1;

  uint8_t* qempty = reinterpret_cast<uint8_t*>(plan + L.qempty_off);
  int32_t* row_act = plan + L.row_act_off;
  const int64_t nqrows = (int64_t)L.ngroups * L.nq;
  for (int64_t r = tid; r < nqrows; r += nthreads) {
    const int g = (int)(r / L.nq), i = (int)(r % L.nq);
    const int jmax = L.causal ? i : L.nq - 1;
    int cnt = 0;
    for (int j = 0; j <= jmax; ++j) cnt += mask_at(mask, L, g, i, j);
    qempty[r] = cnt ? 0 : 1;
    row_act[r] = cnt;
  }
  if (!L.has_csr) return;
  int32_t* frow = plan + L.f_rowptr_off;
  int32_t* brow = plan + L.b_rowptr_off;
  int32_t* jcnt = plan + L.jcnt_off;
  for (int64_t r = tid; r < L.nrows; r += nthreads) {
    const int g = (int)(r / L.npairs), t = (int)(r % L.npairs);
    int nf = 0, nb = 0, j0 = 0, j1 = 0;
    for (int c = 0; c < L.n64; ++c) {
      const int32_t f = fwd_flags(mask, L, g, t, c);
      nf += f != 0;
      j0 += (f & kFlagActive0) != 0;
      j1 += (f & kFlagActive1) != 0;
      nb += bwd_flags(mask, L, g, t, c) != 0;
    }
    frow[r + 1] = nf;
    brow[r + 1] = nb;
    jcnt[(int64_t)g * L.n64 + 2 * t] = j0;
    if (2 * t + 1 < L.n64) jcnt[(int64_t)g * L.n64 + 2 * t + 1] = j1;
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

__global__ void plan_scan_kernel(PlanLayout L, const int32_t* __restrict__ units, int32_t n_units,
                                 int32_t* __restrict__ plan) {
  const int warp = threadIdx.x >> 5;
  int64_t f_nnz = 0, b_nnz = 0;
  if (L.has_csr) {
    if (warp == 0) f_nnz = warp_scan_rowptr(plan + L.f_rowptr_off, L.nrows);
    if (warp == 1) b_nnz = warp_scan_rowptr(plan + L.b_rowptr_off, L.nrows);
  }
  if (units) {
    uint8_t* usel = reinterpret_cast<uint8_t*>(plan + L.usel_off);
    for (int i = threadIdx.x; i < n_units; i += blockDim.x) {
      const int u = units[i];
      if (u >= 0 && u < L.B * L.H)
        usel[u] = 1;
      else
        record_device_error(DEV_ERR_BOUNDS, 0x500);   // an invalid unit id is left out
    }
  }
  if (threadIdx.x == 0) plan[H_F_NNZ] = (int32_t)f_nnz;
  if (threadIdx.x == 32) plan[H_B_NNZ] = (int32_t)b_nnz;
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

// ------------------------------------------------------------------------------ work kernel
constexpr int kWorkThreads = 1024;

// Block-wide sum of a 64-bit value (all threads of the block call it; result on all threads).
__device__ long long block_sum(long long v, long long* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  long long s = 0;
  for (int w = 0; w < (int)(blockDim.x >> 5); ++w) s += red[w];
  __syncthreads();
  return s;
}

// Block-wide exclusive scan over n values produced by f(i) (three int32 components at once);
// g(i, exclusive prefix) is called for every i.  Deterministic.
template <class F, class G>
__device__ void block_scan3(int n, F f, G g, int3* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  int3 carry = make_int3(0, 0, 0);
  for (int base = 0; base < n; base += blockDim.x) {
    const int i = base + threadIdx.x;
    const int3 v = i < n ? f(i) : make_int3(0, 0, 0);
    int3 s = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int x = __shfl_up_sync(0xffffffffu, s.x, o), y = __shfl_up_sync(0xffffffffu, s.y, o),
                z = __shfl_up_sync(0xffffffffu, s.z, o);
      if (lane >= o) { s.x += x; s.y += y; s.z += z; }
    }
    if (lane == 31) red[warp] = s;
    __syncthreads();
    int3 wpre = carry;
    int3 tot = carry;
    for (int w = 0; w < nw; ++w) {
      if (w < warp) { wpre.x += red[w].x; wpre.y += red[w].y; wpre.z += red[w].z; }
      tot.x += red[w].x; tot.y += red[w].y; tot.z += red[w].z;
    }
    if (i < n) g(i, make_int3(wpre.x + s.x - v.x, wpre.y + s.y - v.y, wpre.z + s.z - v.z));
    __syncthreads();
    carry = tot;
  }
}

// Stable order of n indices by descending cost (0..maxc) by one warp: out[pos] = index.
template <class C>
__device__ void warp_sort_desc(int n, int maxc, C cost_of, int32_t* out, int32_t* hist /* maxc + 2 */) {
  const int lane = threadIdx.x & 31;
  for (int c = lane; c <= maxc + 1; c += 32) hist[c] = 0;
  __syncwarp();
  for (int base = 0; base < n; base += 32) {
    const int i = base + lane;
    const int c = (i < n) ? cost_of(i) : -1;
    const unsigned grp = __match_any_sync(0xffffffffu, c);
    if (c >= 0 && lane == __ffs(grp) - 1) hist[c] += __popc(grp);
    __syncwarp();
  }
  if (lane == 0) {  // bucket bases, largest cost first
    int32_t acc = 0;
    for (int c = maxc; c >= 0; --c) {
      const int32_t k = hist[c];
      hist[c] = acc;
      acc += k;
    }
  }
  __syncwarp();
  for (int base = 0; base < n; base += 32) {
    const int i = base + lane;
    const int c = (i < n) ? cost_of(i) : -1;
    const unsigned grp = __match_any_sync(0xffffffffu, c);
    const int rank = __popc(grp & ((1u << lane) - 1u));
    if (c >= 0) out[hist[c] + rank] = i;
    __syncwarp();
    if (c >= 0 && lane == __ffs(grp) - 1) hist[c] += __popc(grp);
    __syncwarp();
  }
}

__global__ void __launch_bounds__(kWorkThreads) plan_work_kernel(PlanLayout L, int32_t* __restrict__ plan,
                                                                 int32_t workers, int32_t pairing) {
  extern __shared__ int32_t smem[];   // 2 * (n64 + 2) histogram words
  __shared__ long long s_red[32];
  __shared__ int3 s_red3[32];
  __shared__ int s_nsel;
  const int tid = threadIdx.x, warp = tid >> 5;
  const uint8_t* usel = reinterpret_cast<const uint8_t*>(plan + L.usel_off);
  int32_t* sel = plan + L.sel_off;
  int32_t* grp_sel = plan + L.grp_sel_off;
  int32_t* grp_off = plan + L.grp_off_off;
  int32_t* grp_poff = plan + L.grp_poff_off;
  const int U = plan_pair_units(L.B, L.H, L.Bm, L.Hm);

  // 1. Selected-unit lists (serial, O(B * H)).
  if (tid == 0) {
    int n = 0;
    for (int u = 0; u < L.B * L.H; ++u)
      if (usel[u]) sel[n++] = u;
    s_nsel = n;
    int k = 0, pk = 0;
    for (int g = 0; g < L.ngroups; ++g) {
      grp_off[g] = k;
      grp_poff[g] = pk;
      const int k0 = k;
      for (int m = 0; m < U; ++m) {
        const int u = unit_in_group(L, g, m);
        if (usel[u]) grp_sel[k++] = u;
      }
      pk += (k - k0 + 1) / 2;
    }
    grp_off[L.ngroups] = k;
    grp_poff[L.ngroups] = pk;
  }
  __syncthreads();
  const int nsel = s_nsel;
  auto group_of_unit = [&](int u) { return L.group_of(u / L.H, u % L.H); };

  // 2. Statistics over the selected units.
  const int32_t* row_act = plan + L.row_act_off;
  const uint8_t* qempty = reinterpret_cast<const uint8_t*>(plan + L.qempty_off);
  long long act = 0, emp = 0;
  for (int64_t i = tid; i < (int64_t)nsel * L.nq; i += blockDim.x) {
    const int g = group_of_unit(sel[i / L.nq]);
    const int64_t r = (int64_t)g * L.nq + i % L.nq;
    act += row_act[r];
    emp += qempty[r];
  }
  const long long active = block_sum(act, s_red);
  const long long empty = block_sum(emp, s_red);

  long long tiles = 0, useful = 0;
  int fwd_pair = 0, n_work = 0, n_split = 0, n_slots = 0, cap = 0;
  if (L.has_csr) {
    const int32_t* frow = plan + L.f_rowptr_off;
    const int32_t* brow = plan + L.b_rowptr_off;
    const int32_t* fent = plan + L.f_entries_off;
    const int32_t* jcnt = plan + L.jcnt_off;
    const int nsel_items = nsel * L.npairs;

    // 3. Backward (and dQ) items of the selected units, longest first.
    if (warp < 2) {
      const int32_t* rp = warp == 0 ? frow : brow;
      int32_t* items = plan + (warp == 0 ? L.f_items_off : L.b_items_off);
      int32_t* hist = smem + warp * (L.n64 + 2);
      auto cost = [&](int i) {
        const int r = group_of_unit(sel[i / L.npairs]) * L.npairs + i % L.npairs;
        return rp[r + 1] - rp[r];
      };
      warp_sort_desc(nsel_items, L.n64, cost, items, hist);
      // warp_sort_desc wrote positions as indices into the selected list; re-encode as unit items.
      __syncwarp();
      for (int i = threadIdx.x & 31; i < nsel_items; i += 32) {
        const int x = items[i];
        items[i] = sel[x / L.npairs] * L.npairs + x % L.npairs;
      }
    }

    // 4. Forward pairing: the same query chunk of two units that share the mask when such
    // units exist and pairing query chunks 2t, 2t+1 would leave more than 12% of the 64-row
    // halves it computes masked out (measured crossover: 67-80% useful halves favour unit
    // pairing by 3-8%, 98.5% favours query-chunk pairing by 7%).
    long long ent = 0, use = 0;
    for (int i = tid; i < nsel; i += blockDim.x) {
      const int g = group_of_unit(sel[i]);
      ent += frow[(g + 1) * L.npairs] - frow[g * L.npairs];
      for (int j = 0; j < L.n64; ++j) use += jcnt[(int64_t)g * L.n64 + j];
    }
    const long long entries = block_sum(ent, s_red);
    useful = block_sum(use, s_red);
    bool pairs_possible = false;
    for (int g = 0; g < L.ngroups && !pairs_possible; ++g) pairs_possible = grp_off[g + 1] - grp_off[g] >= 2;
    const int32_t auto_pair = (pairs_possible && 100 * useful < 88 * (2 * entries)) ? kPairUnits : kPairQuery;
    fwd_pair = pairing == XSAKE_PAIRING_QUERY ? kPairQuery : pairing == XSAKE_PAIRING_UNITS ? kPairUnits : auto_pair;
    const bool units = fwd_pair == kPairUnits;
    tiles = units ? useful : 2 * entries;

    // 5. Base work items and their steps (kv chunks walked).
    const int PT = grp_poff[L.ngroups];
    const int n_base = units ? L.n64 * PT : nsel_items;
    int32_t* base_cost = plan + L.f_order_off;   // reused by the final sort below
    auto describe = [&](int i, FWork& w, int& row) {
      if (units) {
        const int jj = i / PT, rem = i % PT;
        const int j = L.n64 - 1 - jj;
        int lo = 0, hi = L.ngroups - 1;   // group g with grp_poff[g] <= rem < grp_poff[g + 1]
        while (lo < hi) {
          const int mid = (lo + hi + 1) >> 1;
          if (grp_poff[mid] <= rem) lo = mid; else hi = mid - 1;
        }
        const int g = lo, p = rem - grp_poff[g], cnt = grp_off[g + 1] - grp_off[g];
        w.u0 = grp_sel[grp_off[g] + 2 * p];
        w.u1 = (2 * p + 1 < cnt) ? grp_sel[grp_off[g] + 2 * p + 1] : -1;
        w.q = j;
        row = g * L.npairs + (j >> 1);
        return jcnt[(int64_t)g * L.n64 + j];
      }
      const int u = sel[i / L.npairs], t = i % L.npairs;
      w.u0 = u;
      w.u1 = -1;
      w.q = t;
      row = group_of_unit(u) * L.npairs + t;
      return frow[row + 1] - frow[row];
    };
    long long tot = 0;
    for (int i = tid; i < n_base; i += blockDim.x) {
      FWork w;
      int row;
      const int c = describe(i, w, row);
      base_cost[i] = c;
      tot += c;
    }
    const long long total = block_sum(tot, s_red);

    // 6. Piece size: at least 3/4 of the average steps per worker (so a job that fills the
    // GPU many times over is not split), at least kMinPieceSteps, at most kMaxPieces pieces
    // per item, and grown until the split pieces fit the kSplitSlots partial slots.
    const int W = workers > 0 ? workers : 1;
    int cap0 = (int)((3 * total + 4ll * W - 1) / (4ll * W));
    cap0 = max(cap0, kMinPieceSteps);
    cap0 = max(cap0, (L.n64 + kMaxPieces - 1) / kMaxPieces);
    int lo_c = cap0, hi_c = max(cap0, L.n64);
    while (lo_c < hi_c) {   // smallest cap whose pieces fit the slots (uniform across the block)
      const int mid = (lo_c + hi_c) >> 1;
      long long need = 0;
      for (int i = tid; i < n_base; i += blockDim.x) {
        const int c = base_cost[i];
        if (c > mid) need += (c + mid - 1) / mid;
      }
      need = block_sum(need, s_red);
      if (need <= kSplitSlots) hi_c = mid; else lo_c = mid + 1;
    }
    cap = lo_c;

    // 7. Pieces of every item: scan (pieces, split groups, slots), then write them unsorted.
    FWork* tmp = reinterpret_cast<FWork*>(plan + L.f_tmp_off);
    int32_t* piece_cost = plan + L.f_cost_off;
    auto pieces_of = [&](int c) { return c > cap ? (c + cap - 1) / cap : 1; };
    block_scan3(
        n_base,
        [&](int i) {
          const int n = pieces_of(base_cost[i]);
          return make_int3(n, n > 1 ? 1 : 0, n > 1 ? n : 0);
        },
        [&](int i, int3 pre) {
          FWork w;
          int row;
          const int c = describe(i, w, row);
          const int n = pieces_of(c);
          const int rowcnt = frow[row + 1] - frow[row];
          const int32_t fa = (w.q & 1) ? kFlagActive1 : kFlagActive0;
          const int32_t* e = fent + frow[row];
          for (int k = 0; k < n; ++k) {
            FWork x = w;
            const int per = c / n, extra = c % n;
            const int s0 = k * per + min(k, extra), s1 = s0 + per + (k < extra ? 1 : 0);
            x.parts = (k << 8) | n;
            x.grp = n > 1 ? pre.y : -1;
            x.slot = n > 1 ? pre.z : 0;
            if (n == 1) {
              x.lo = 0;
              x.hi = rowcnt;
            } else if (!units) {      // every entry of a pair row is a step of its tile
              x.lo = s0;
              x.hi = s1;
            } else {                  // steps are the entries half j % 2 attends
              int cnt = 0, lo = rowcnt, hi = rowcnt;
              for (int r = 0; r < rowcnt; ++r) {
                if (!(e[r] & fa)) continue;
                if (cnt == s0) lo = r;
                if (cnt == s1) { hi = r; break; }
                ++cnt;
              }
              x.lo = lo;
              x.hi = hi;
            }
            x.lo += frow[row];   // absolute positions in f_entries: no row lookup when decoding
            x.hi += frow[row];
            tmp[pre.x + k] = x;
            piece_cost[pre.x + k] = s1 - s0;
          }
        },
        s_red3);
    long long np = 0, ns = 0, nsl = 0;
    for (int i = tid; i < n_base; i += blockDim.x) {
      const int n = pieces_of(base_cost[i]);
      np += n;
      ns += n > 1;
      nsl += n > 1 ? n : 0;
    }
    n_work = (int)block_sum(np, s_red);
    n_split = (int)block_sum(ns, s_red);
    n_slots = (int)block_sum(nsl, s_red);

    // 8. Order.  Unit pairing: the enumeration order (query chunk j descending, i.e. longest
    // first under a causal mask, each split item's pieces in place); measured 1.5% faster on
    // HADS masks than a strict sort by steps, which interleaves heads.  Query-chunk pairing:
    // longest first by steps (stable).
    __syncthreads();
    int32_t* order = plan + L.f_order_off;
    if (units) {
      for (int i = tid; i < n_work; i += blockDim.x) order[i] = i;
    } else if (warp == 0) {
      warp_sort_desc(n_work, L.n64, [&](int i) { return piece_cost[i]; }, order, smem);
    }
    __syncthreads();
    FWork* work = reinterpret_cast<FWork*>(plan + L.f_work_off);
    for (int i = tid; i < n_work; i += blockDim.x) work[i] = tmp[order[i]];
  }
  __syncthreads();
  if (tid == 0) {
    int32_t* hdr = plan;
    hdr[H_VERSION] = kPlanVersion;
    hdr[H_B] = L.B; hdr[H_H] = L.H; hdr[H_S] = L.S; hdr[H_BM] = L.Bm; hdr[H_HM] = L.Hm;
    hdr[H_BS] = L.bs; hdr[H_CAUSAL] = L.causal; hdr[H_HAS_CSR] = L.has_csr;
    hdr[H_SEL_UNITS] = nsel;
    hdr[H_F_ITEMS] = L.has_csr ? nsel * L.npairs : 0;
    hdr[H_B_ITEMS] = L.has_csr ? nsel * L.npairs : 0;
    hdr[H_F_WORK] = n_work;
    hdr[H_ACTIVE_LO] = (int32_t)(active & 0xffffffff); hdr[H_ACTIVE_HI] = (int32_t)(active >> 32);
    hdr[H_TILES_LO] = (int32_t)(tiles & 0xffffffff);   hdr[H_TILES_HI] = (int32_t)(tiles >> 32);
    hdr[H_EMPTY_LO] = (int32_t)(empty & 0xffffffff);   hdr[H_EMPTY_HI] = (int32_t)(empty >> 32);
    hdr[H_ITEMS_LO] = n_work;                          hdr[H_ITEMS_HI] = 0;
    hdr[H_FWD_PAIR] = fwd_pair;
    hdr[H_SPLIT_GROUPS] = n_split;
    hdr[H_SPLIT_SLOTS] = n_slots;
    hdr[H_SPLIT_CAP] = cap;
    hdr[H_WORKERS] = workers;
    __threadfence();
    hdr[H_MAGIC] = kPlanMagic;
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
  XSAKE_REQUIRE((int64_t)d->batch * d->heads * ((d->seq / 64 + 2) / 2) < (1ll << 30),
                XSAKE_EUNSUPPORTED, "too many work items");
  XSAKE_REQUIRE((int64_t)d->batch * d->heads * (d->seq / 64 + 1) < (1ll << 30), XSAKE_EUNSUPPORTED,
                "too many work items");
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

extern "C" int xsake_mask_compile_ex(const XsakeMaskDims* dims, const XsakePlanOptions* opt, const uint8_t* mask_dev,
                                     void* plan_dev, size_t plan_bytes, void* stream) {
  clear_error();
  PlanLayout L;
  int st = plan_layout_from_dims(dims, &L);
  if (st) return st;
  XSAKE_REQUIRE(mask_dev && plan_dev, XSAKE_EINVAL, "mask and plan must be device pointers");
  XSAKE_REQUIRE(plan_bytes >= (size_t)L.total_words * 4, XSAKE_EINVAL,
                "plan buffer too small: %zu < %lld bytes", plan_bytes, (long long)L.total_words * 4);
  XSAKE_REQUIRE(((uintptr_t)plan_dev & 15) == 0, XSAKE_EINVAL, "plan must be 16-byte aligned");
  const int32_t* units = nullptr;
  int32_t n_units = 0, workers = 0, pairing = XSAKE_PAIRING_AUTO;
  if (opt) {
    units = opt->units_dev;
    n_units = opt->n_units;
    workers = opt->workers;
    pairing = opt->forward_pairing;
    XSAKE_REQUIRE(pairing >= XSAKE_PAIRING_AUTO && pairing <= XSAKE_PAIRING_UNITS, XSAKE_EINVAL,
                  "forward_pairing %d is not one of XSAKE_PAIRING_*", pairing);
    XSAKE_REQUIRE(units != nullptr || n_units == 0, XSAKE_EINVAL, "n_units %d without a unit list", n_units);
    XSAKE_REQUIRE(units == nullptr || (n_units > 0 && n_units <= dims->batch * dims->heads), XSAKE_EINVAL,
                  "n_units %d must be in [1, batch * heads = %d]", n_units, dims->batch * dims->heads);
    XSAKE_REQUIRE(workers >= 0, XSAKE_EINVAL, "workers %d must be >= 0", workers);
  }
  DeviceInfo di;
  if ((st = device_info(&di))) return st;
  if (workers == 0) workers = 2 * di.sm_count;   // two tile workers per SM in the forward kernel
  cudaStream_t s = as_stream(stream);
  const int64_t work = std::max<int64_t>((int64_t)L.ngroups * L.nq * L.nq, 3 * (int64_t)L.nrows);
  const int blocks = (int)std::min<int64_t>((work + 255) / 256, 4 * (int64_t)di.sm_count);
  plan_rows_kernel<<<std::max(blocks, 1), 256, 0, s>>>(L, mask_dev, units, (int32_t*)plan_dev);
  if ((st = check_launch("plan_rows_kernel"))) return st;
  plan_scan_kernel<<<1, 1024, 0, s>>>(L, units, n_units, (int32_t*)plan_dev);
  if ((st = check_launch("plan_scan_kernel"))) return st;
  if (L.has_csr) {
    const int fb = (int)std::min<int64_t>((3 * (int64_t)L.nrows + 127) / 128, 4 * (int64_t)di.sm_count);
    plan_fill_kernel<<<std::max(fb, 1), 128, 0, s>>>(L, (int32_t*)plan_dev);
    if ((st = check_launch("plan_fill_kernel"))) return st;
  }
  const size_t smem = 2 * (size_t)(L.n64 + 2) * sizeof(int32_t);
  XSAKE_REQUIRE(smem <= 48 * 1024, XSAKE_EUNSUPPORTED, "seq too long for the plan compiler");
  plan_work_kernel<<<1, kWorkThreads, smem, s>>>(L, (int32_t*)plan_dev, workers, pairing);
  return check_launch("plan_work_kernel");
}

extern "C" int xsake_mask_compile(const XsakeMaskDims* dims, const uint8_t* mask_dev, void* plan_dev,
                                  size_t plan_bytes, void* stream) {
  return xsake_mask_compile_ex(dims, nullptr, mask_dev, plan_dev, plan_bytes, stream);
}

extern "C" int xsake_mask_plan_info(const void* plan_dev, void* stream, XsakePlanInfo* info) {
  clear_error();
  XSAKE_REQUIRE(plan_dev && info, XSAKE_EINVAL, "NULL argument");
  int32_t hdr[kPlanHeaderWords];
  cudaStream_t s = as_stream(stream);
  XSAKE_CUDA_TRY(cudaMemcpyAsync(hdr, plan_dev, sizeof(hdr), cudaMemcpyDeviceToHost, s));
  XSAKE_CUDA_TRY(cudaStreamSynchronize(s));
  XSAKE_REQUIRE(hdr[H_MAGIC] == kPlanMagic && hdr[H_VERSION] == kPlanVersion, XSAKE_EINVAL, "not a compiled plan");
  auto u64 = [&](int lo) { return (int64_t)(uint32_t)hdr[lo] | ((int64_t)hdr[lo + 1] << 32); };
  info->active_blocks = u64(H_ACTIVE_LO);
  info->computed_tiles = u64(H_TILES_LO);
  info->empty_qblocks = u64(H_EMPTY_LO);
  info->work_items = hdr[H_F_WORK];
  info->selected_units = hdr[H_SEL_UNITS];
  info->pairing = hdr[H_FWD_PAIR];
  info->split_items = hdr[H_SPLIT_GROUPS];
  info->split_slots = hdr[H_SPLIT_SLOTS];
  info->split_cap = hdr[H_SPLIT_CAP];
  info->workers = hdr[H_WORKERS];
  return XSAKE_OK;
}

extern "C" int xsake_mask_plan_stats(const void* plan_dev, void* stream, int64_t out[4]) {
  XSAKE_REQUIRE(out != nullptr, XSAKE_EINVAL, "NULL argument");
  XsakePlanInfo info;
  int st = xsake_mask_plan_info(plan_dev, stream, &info);
  if (st) return st;
  out[0] = info.active_blocks;
  out[1] = info.computed_tiles;
  out[2] = info.empty_qblocks;
  out[3] = info.work_items;
  return XSAKE_OK;
}
