// HADS calibration: per-head Shannon entropy of materialised attention probabilities.
// Replaces compute_attention_entropy (kernels/hads/hads_pattern.py:36-50):
//   H[b,h,q] = -sum_k clip(p,1e-9,1) * log(clip(p,1e-9,1)),  reduced over (b, q) per head.
// HBM-bound: every probability is read once with 16-byte loads; each warp owns one row and
// reduces it with shuffles; rows are summed in fp64 in a fixed order (per-CTA partials in the
// workspace, then one pass per head), so the result is bitwise reproducible.
#include "common.cuh"

#include <algorithm>
#include <mutex>

XSAKE_DEFINE_DEVICE_ERROR(entropy)

namespace xsake {
namespace {

constexpr int kEntWarps = 8;
constexpr float kClipLo = 1e-9f;

__device__ __forceinline__ float plogp(float p) {
  p = fminf(fmaxf(p, kClipLo), 1.0f);
  return p * __log2f(p);
}

struct EntropyGeom {
  int64_t B, H, Sq, Sk;
  int64_t rows_per_cta;   // divides Sq so a CTA never straddles two (b, h) slices
  int64_t ctas_per_bh;
};

// Work is cut into chunks of rows_per_cta (<= 16) consecutive rows of one (b, h) slice; chunk c
// writes partial[c].  A persistent grid gives each CTA a contiguous, balanced range of chunks;
// each warp reduces two rows of a chunk with all their loads issued up front (eight 16-byte
// words per row per lane when Sk = 1024), and the chunk's rows are summed in a fixed order, so
// the partials do not depend on the grid.
__global__ void __launch_bounds__(256) entropy_rows_kernel(const float* __restrict__ p, EntropyGeom g,
                                                           int64_t nchunks, double* __restrict__ partial) {
  __shared__ double srow[2][16];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t c0 = nchunks * blockIdx.x / gridDim.x, c1 = nchunks * (blockIdx.x + 1) / gridDim.x;
  int it = 0;
  for (int64_t c = c0; c < c1; ++c, ++it) {
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
      const int r = 2 * warp + rr;
      double ent = 0.0;
      if (r < g.rows_per_cta) {
        const float* pr = p + (c * g.rows_per_cta + r) * g.Sk;
        float s = 0.f;
        if (g.Sk == 1024) {
          const float4* p4 = reinterpret_cast<const float4*>(pr);
          float4 t[8];
#pragma unroll
          for (int u = 0; u < 8; ++u) t[u] = p4[lane + 32 * u];
#pragma unroll
          for (int u = 0; u < 8; ++u) s += plogp(t[u].x) + plogp(t[u].y) + plogp(t[u].z) + plogp(t[u].w);
        } else if ((g.Sk % 4) == 0) {
          const float4* p4 = reinterpret_cast<const float4*>(pr);
          for (int64_t v = lane; v < g.Sk / 4; v += 32) {
            const float4 a = p4[v];
            s += plogp(a.x) + plogp(a.y) + plogp(a.z) + plogp(a.w);
          }
        } else {
          for (int64_t k = lane; k < g.Sk; k += 32) s += plogp(pr[k]);
        }
        s = warp_sum(s);
        ent = -(double)s * (double)kLn2;
      }
      if (lane == 0) srow[it & 1][r] = ent;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      double t = 0.0;
      for (int r = 0; r < g.rows_per_cta; ++r) t += srow[it & 1][r];
      partial[c] = t;
    }
  }
}

// One CTA per head: thread t sums partials t, t + 256, ... of the head's B * ctas_per_bh (in
// (b, chunk) order), then a fixed shared-memory tree; the order depends only on the shapes.
__global__ void __launch_bounds__(256) entropy_heads_kernel(const double* __restrict__ partial, EntropyGeom g,
                                                            double* __restrict__ head_sums) {
  __shared__ double red[256];
  const int h = blockIdx.x;
  const int64_t per_b = g.ctas_per_bh, n = g.B * per_b;
  double t = 0.0;
  for (int64_t i = threadIdx.x; i < n; i += 256) {
    const int64_t b = i / per_b, c = i - b * per_b;
    t += partial[(b * g.H + h) * per_b + c];
  }
  red[threadIdx.x] = t;
  __syncthreads();
  for (int w = 128; w > 0; w >>= 1) {
    if ((int)threadIdx.x < w) red[threadIdx.x] += red[threadIdx.x + w];
    __syncthreads();
  }
  if (threadIdx.x == 0) head_sums[h] = red[0];
}

// One wave: as many CTAs as are resident at once (occupancy of this kernel), so no CTA starts
// after the others have drained and every SM streams until the end.
unsigned entropy_grid(int64_t nchunks) {
  DeviceInfo di;
  const int sms = device_info(&di) == XSAKE_OK ? di.sm_count : 148;
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, entropy_rows_kernel, 256, 0) != cudaSuccess || per_sm < 1)
    per_sm = 1;
  clear_error();
  return (unsigned)std::max<int64_t>(1, std::min<int64_t>(nchunks, (int64_t)sms * per_sm));
}

EntropyGeom geom(int64_t B, int64_t H, int64_t Sq, int64_t Sk) {
  EntropyGeom g{B, H, Sq, Sk, 1, 1};
  // Chunks of up to 16 rows (a divisor of Sq), two rows per warp.
  int64_t rpc = 1;
  for (int64_t c = std::min<int64_t>(16, Sq); c >= 1; --c)
    if (Sq % c == 0) { rpc = c; break; }
  g.rows_per_cta = rpc;
  g.ctas_per_bh = Sq / rpc;
  return g;
}

}  // namespace
}  // namespace xsake

using namespace xsake;

extern "C" int xsake_entropy_workspace_size(int64_t batch, int64_t heads, int64_t sq, size_t* bytes) {
  clear_error();
  XSAKE_REQUIRE(bytes && batch > 0 && heads > 0 && sq > 0, XSAKE_EINVAL, "bad arguments");
  const EntropyGeom g = geom(batch, heads, sq, 1);
  *bytes = (size_t)(batch * heads * g.ctas_per_bh) * sizeof(double);
  return XSAKE_OK;
}

extern "C" int xsake_entropy_rows(const float* p_dev, int64_t batch, int64_t heads, int64_t sq, int64_t sk,
                                  double* head_sums_dev, void* workspace_dev, size_t workspace_bytes,
                                  void* stream) {
  clear_error();
  XSAKE_REQUIRE(batch > 0 && heads > 0 && sq > 0 && sk > 0, XSAKE_EINVAL, "dims must be positive");
  XSAKE_REQUIRE(p_dev && head_sums_dev, XSAKE_EINVAL, "NULL pointer");
  XSAKE_REQUIRE(((uintptr_t)p_dev & 15) == 0, XSAKE_EINVAL, "p must be 16-byte aligned");
  const EntropyGeom g = geom(batch, heads, sq, sk);
  const int64_t nctas = batch * heads * g.ctas_per_bh;
  XSAKE_REQUIRE(nctas < (1ll << 31), XSAKE_EUNSUPPORTED, "too many rows");
  XSAKE_REQUIRE(workspace_dev && workspace_bytes >= (size_t)nctas * sizeof(double), XSAKE_EINVAL,
                "workspace too small: %zu < %zu bytes", workspace_bytes, (size_t)nctas * sizeof(double));
  cudaStream_t s = as_stream(stream);
  double* partial = reinterpret_cast<double*>(workspace_dev);
  entropy_rows_kernel<<<entropy_grid(nctas), 256, 0, s>>>(p_dev, g, nctas, partial);
  int st = check_launch("entropy_rows_kernel");
  if (st) return st;
  entropy_heads_kernel<<<(unsigned)heads, 256, 0, s>>>(partial, g, head_sums_dev);
  return check_launch("entropy_heads_kernel");
}

// ------------------------------------------------------------------------------------------
// Allocation-free variant of xsake_entropy_rows.
//
// Some callers cannot hand this library a device workspace and cannot allocate one either:
// a framework plugin (for example an XLA FFI handler) must take every byte of device memory
// from its framework's allocator, and a process whose memory is fully reserved by a pool
// allocator would see a raw cudaMalloc fail; cudaMalloc also synchronises the device, which
// a latency-critical loop cannot afford.  For them the per-CTA partial sums live in the
// static device array below instead of a workspace.
//
// Limits and behaviour:
//   * at most kNoAllocMaxPartials = 65,536 partial sums (512 KiB, held by every GPU that loads
//     the library until the process exits): batch * heads * ctas_per_slice must not exceed it,
//     where ctas_per_slice = seq_q / (largest divisor of seq_q that is <= 16); larger calls are
//     rejected with XSAKE_EUNSUPPORTED before anything is launched;
//   * the first call on each device looks up the array's device address with
//     cudaGetSymbolAddress (with that device current); make that first call before any stream
//     capture begins;
//   * all calls share the one array: calls that overlap on the GPU (concurrent streams) race
//     and corrupt each other's results; calls ordered on one stream are fine;
//   * the array keeps the previous call's contents; nothing needs clearing because every slot a
//     call reads is first written by the same call.
namespace xsake {
namespace {

constexpr int64_t kNoAllocMaxPartials = 65536;
static __device__ __align__(256) double g_entropy_partials[kNoAllocMaxPartials];

constexpr int kNoAllocMaxDevices = 64;
double* g_partials_ptr[kNoAllocMaxDevices];
cudaError_t g_partials_err[kNoAllocMaxDevices];
std::once_flag g_partials_once[kNoAllocMaxDevices];

int partials_address(double** out) {
  int dev = 0;
  XSAKE_CUDA_TRY(cudaGetDevice(&dev));
  XSAKE_REQUIRE(dev >= 0 && dev < kNoAllocMaxDevices, XSAKE_EUNSUPPORTED, "device ordinal %d", dev);
  std::call_once(g_partials_once[dev], [dev] {
    g_partials_err[dev] = cudaGetSymbolAddress(reinterpret_cast<void**>(&g_partials_ptr[dev]), g_entropy_partials);
  });
  XSAKE_REQUIRE(g_partials_err[dev] == cudaSuccess, XSAKE_ECUDA, "cudaGetSymbolAddress failed on device %d: %s", dev,
                cudaGetErrorString(g_partials_err[dev]));
  *out = g_partials_ptr[dev];
  return XSAKE_OK;
}

}  // namespace
}  // namespace xsake

extern "C" int xsake_entropy_rows_noalloc(const float* p_dev, int64_t batch, int64_t heads, int64_t sq, int64_t sk,
                                          double* head_sums_dev, void* stream) {
  clear_error();
  XSAKE_REQUIRE(batch > 0 && heads > 0 && sq > 0 && sk > 0, XSAKE_EINVAL, "dims must be positive");
  XSAKE_REQUIRE(p_dev && head_sums_dev, XSAKE_EINVAL, "NULL pointer");
  XSAKE_REQUIRE(((uintptr_t)p_dev & 15) == 0, XSAKE_EINVAL, "p must be 16-byte aligned");
  const EntropyGeom g = geom(batch, heads, sq, sk);
  const int64_t nctas = batch * heads * g.ctas_per_bh;
  XSAKE_REQUIRE(nctas <= kNoAllocMaxPartials, XSAKE_EUNSUPPORTED,
                "xsake_entropy_rows_noalloc: %lld partial sums exceed its static limit of %lld "
                "(batch * heads * ctas_per_slice); use xsake_entropy_rows with a workspace",
                (long long)nctas, (long long)kNoAllocMaxPartials);
  double* partial = nullptr;
  int st = partials_address(&partial);
  if (st) return st;
  cudaStream_t s = as_stream(stream);
  entropy_rows_kernel<<<entropy_grid(nctas), 256, 0, s>>>(p_dev, g, nctas, partial);
  if ((st = check_launch("entropy_rows_kernel"))) return st;
  entropy_heads_kernel<<<(unsigned)heads, 256, 0, s>>>(partial, g, head_sums_dev);
  return check_launch("entropy_heads_kernel");
}
