/*
 * A caller of libxsake_hads.so with no Python and no PyTorch: the way a JAX FFI handler or a C++
 * trainer binds the C ABI.  It reads its inputs from a binary file, owns device memory through the
 * CUDA runtime, compiles a block-mask plan, runs the attention forward, softmax and LayerNorm on
 * one stream, and writes the outputs to a binary file.
 *
 * Input file (little endian): int32 B, H, S, D, block, causal, mask_heads, rows, cols, ln_rows, ln_d;
 * then float32 q, k, v [B, H, S, D] (converted to bf16 here), uint8 mask [mask_heads, nb, nb],
 * float32 softmax input [rows, cols], float32 LayerNorm x [ln_rows, ln_d], gamma [ln_d], beta [ln_d].
 * Output file: float32 attention output [B, H, S, D] and lse [B, H, S], softmax [rows, cols],
 * LayerNorm [ln_rows, ln_d].
 *
 * usage: xsake_c_client in.bin out.bin
 */
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "xsake_hads.h"

#define CK(x) do { cudaError_t e_ = (x); if (e_ != cudaSuccess) { fprintf(stderr, "%s: %s\n", #x, cudaGetErrorString(e_)); return 2; } } while (0)
#define XK(x) do { int s_ = (x); if (s_ != XSAKE_OK) { fprintf(stderr, "%s: status %d: %s\n", #x, s_, xsake_last_error()); return 3; } } while (0)

static void* read_all(FILE* f, size_t n) {
  void* p = malloc(n ? n : 1);
  if (p && n && fread(p, 1, n, f) != n) { free(p); return NULL; }
  return p;
}

int main(int argc, char** argv) {
  if (argc != 3) { fprintf(stderr, "usage: %s in.bin out.bin\n", argv[0]); return 1; }
  FILE* f = fopen(argv[1], "rb");
  if (!f) { perror(argv[1]); return 1; }
  int32_t hd[11];
  if (fread(hd, sizeof(int32_t), 11, f) != 11) { fprintf(stderr, "short header\n"); return 1; }
  const int B = hd[0], H = hd[1], S = hd[2], D = hd[3], bs = hd[4], causal = hd[5], Hm = hd[6];
  const int64_t rows = hd[7], cols = hd[8], ln_rows = hd[9], ln_d = hd[10];
  const size_t n_qkv = (size_t)B * H * S * D, nb = (size_t)(S / bs);
  float* q = (float*)read_all(f, n_qkv * 4);
  float* k = (float*)read_all(f, n_qkv * 4);
  float* v = (float*)read_all(f, n_qkv * 4);
  uint8_t* mask = (uint8_t*)read_all(f, (size_t)Hm * nb * nb);
  float* sx = (float*)read_all(f, (size_t)rows * cols * 4);
  float* lx = (float*)read_all(f, (size_t)ln_rows * ln_d * 4);
  float* lg = (float*)read_all(f, (size_t)ln_d * 4);
  float* lb = (float*)read_all(f, (size_t)ln_d * 4);
  fclose(f);
  if (!q || !k || !v || !mask || !sx || !lx || !lg || !lb) { fprintf(stderr, "short input\n"); return 1; }
  if (xsake_abi_version() != XSAKE_ABI_VERSION) { fprintf(stderr, "ABI version mismatch\n"); return 1; }

  cudaStream_t st;
  CK(cudaStreamCreate(&st));
  /* bf16 q, k, v on the device */
  __nv_bfloat16* hb = (__nv_bfloat16*)malloc(3 * n_qkv * sizeof(__nv_bfloat16));
  for (size_t i = 0; i < n_qkv; ++i) {
    hb[i] = __float2bfloat16(q[i]);
    hb[n_qkv + i] = __float2bfloat16(k[i]);
    hb[2 * n_qkv + i] = __float2bfloat16(v[i]);
  }
  void *dqkv, *dout, *dmask, *dplan, *dws;
  float* dlse;
  CK(cudaMalloc(&dqkv, 3 * n_qkv * 2));
  CK(cudaMalloc(&dout, n_qkv * 2));
  CK(cudaMalloc((void**)&dlse, (size_t)B * H * S * 4));
  CK(cudaMalloc(&dmask, (size_t)Hm * nb * nb));
  CK(cudaMemcpyAsync(dqkv, hb, 3 * n_qkv * 2, cudaMemcpyHostToDevice, st));
  CK(cudaMemcpyAsync(dmask, mask, (size_t)Hm * nb * nb, cudaMemcpyHostToDevice, st));

  XsakeMaskDims dims = {B, H, S, 1, Hm, bs, causal};
  size_t plan_bytes = 0, ws_bytes = 0;
  XK(xsake_mask_plan_bytes(&dims, &plan_bytes));
  CK(cudaMalloc(&dplan, plan_bytes));
  XK(xsake_mask_compile(&dims, (const uint8_t*)dmask, dplan, plan_bytes, st));

  XsakeAttnDesc desc;
  memset(&desc, 0, sizeof(desc));
  desc.dtype = XSAKE_BF16;
  desc.batch = B; desc.heads = H; desc.seq = S; desc.head_dim = D;
  desc.block_size = bs; desc.causal = causal; desc.mask_batch = 1; desc.mask_heads = Hm;
  desc.scale = 0.f;
  const int64_t strides[3] = {(int64_t)H * S * D, (int64_t)S * D, D};
  memcpy(desc.q_stride, strides, sizeof(strides)); memcpy(desc.k_stride, strides, sizeof(strides));
  memcpy(desc.v_stride, strides, sizeof(strides)); memcpy(desc.o_stride, strides, sizeof(strides));
  XK(xsake_attn_fwd_workspace_size(&desc, &ws_bytes));
  CK(cudaMalloc(&dws, ws_bytes));
  char* base = (char*)dqkv;
  XK(xsake_attn_fwd(&desc, dplan, base, base + n_qkv * 2, base + 2 * n_qkv * 2, dout, dlse, dws, ws_bytes, st));

  float *dsx, *dsy, *dlx, *dly, *dlg, *dlb;
  CK(cudaMalloc((void**)&dsx, (size_t)rows * cols * 4)); CK(cudaMalloc((void**)&dsy, (size_t)rows * cols * 4));
  CK(cudaMalloc((void**)&dlx, (size_t)ln_rows * ln_d * 4)); CK(cudaMalloc((void**)&dly, (size_t)ln_rows * ln_d * 4));
  CK(cudaMalloc((void**)&dlg, (size_t)ln_d * 4)); CK(cudaMalloc((void**)&dlb, (size_t)ln_d * 4));
  CK(cudaMemcpyAsync(dsx, sx, (size_t)rows * cols * 4, cudaMemcpyHostToDevice, st));
  CK(cudaMemcpyAsync(dlx, lx, (size_t)ln_rows * ln_d * 4, cudaMemcpyHostToDevice, st));
  CK(cudaMemcpyAsync(dlg, lg, (size_t)ln_d * 4, cudaMemcpyHostToDevice, st));
  CK(cudaMemcpyAsync(dlb, lb, (size_t)ln_d * 4, cudaMemcpyHostToDevice, st));
  XK(xsake_softmax_fwd(XSAKE_F32, rows, cols, dsx, dsy, st));
  XK(xsake_layernorm_fwd(XSAKE_F32, ln_rows, ln_d, dlx, dlg, dlb, 1e-5f, dly, NULL, NULL, st));

  __nv_bfloat16* ho = (__nv_bfloat16*)malloc(n_qkv * 2);
  float* hl = (float*)malloc((size_t)B * H * S * 4);
  float* hs = (float*)malloc((size_t)rows * cols * 4);
  float* hy = (float*)malloc((size_t)ln_rows * ln_d * 4);
  CK(cudaMemcpyAsync(ho, dout, n_qkv * 2, cudaMemcpyDeviceToHost, st));
  CK(cudaMemcpyAsync(hl, dlse, (size_t)B * H * S * 4, cudaMemcpyDeviceToHost, st));
  CK(cudaMemcpyAsync(hs, dsy, (size_t)rows * cols * 4, cudaMemcpyDeviceToHost, st));
  CK(cudaMemcpyAsync(hy, dly, (size_t)ln_rows * ln_d * 4, cudaMemcpyDeviceToHost, st));
  CK(cudaStreamSynchronize(st));
  int32_t code = 0;
  XK(xsake_device_error(st, &code));
  if (code) { fprintf(stderr, "device error word 0x%08x\n", code); return 4; }

  FILE* g = fopen(argv[2], "wb");
  if (!g) { perror(argv[2]); return 1; }
  for (size_t i = 0; i < n_qkv; ++i) { const float x = __bfloat162float(ho[i]); fwrite(&x, 4, 1, g); }
  fwrite(hl, 4, (size_t)B * H * S, g);
  fwrite(hs, 4, (size_t)rows * cols, g);
  fwrite(hy, 4, (size_t)ln_rows * ln_d, g);
  fclose(g);
  cudaFree(dqkv); cudaFree(dout); cudaFree(dlse); cudaFree(dmask); cudaFree(dplan); cudaFree(dws);
  cudaFree(dsx); cudaFree(dsy); cudaFree(dlx); cudaFree(dly); cudaFree(dlg); cudaFree(dlb);
  cudaStreamDestroy(st);
  printf("ok\n");
  return 0;
}
