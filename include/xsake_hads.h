/*
 * xsake_hads.h -- C ABI of libxsake_hads.so, the sm_100a (B200) implementation of the
 * HADS block-sparse attention path of Hridambiswas/XSAKE.
 *
 * The reference exposes this path as Python/JAX functions; each entry point below names
 * the reference function it replaces (path:line inside the reference project).  A JAX
 * FFI handler, a ctypes stub or a C++ caller binds these symbols directly.
 *
 * Conventions
 *   - Every pointer argument named *_dev is DEVICE memory owned by the caller.
 *   - Calls are stream-ordered on `stream` (a cudaStream_t passed as void*; NULL = the
 *     legacy default stream), never synchronise the host, and never allocate: scratch
 *     comes from a caller-provided workspace whose size the *_workspace_size query gives.
 *   - Return value: XSAKE_OK (0) or an XSAKE_E* code; xsake_last_error() then returns a
 *     message for the calling thread.  Argument errors are detected before any launch.
 *   - Tensors of the attention path use the layout [B, H, S, D] addressed through
 *     element strides (stride of D must be 1), so both [B,H,S,D] and [B,S,H,D] work.
 *   - dtype codes: XSAKE_F32 (float32), XSAKE_BF16 (bfloat16).
 */
#ifndef XSAKE_HADS_H
#define XSAKE_HADS_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define XSAKE_API __attribute__((visibility("default")))
#else
#define XSAKE_API
#endif

#define XSAKE_ABI_VERSION 1

enum {
  XSAKE_OK = 0,
  XSAKE_EINVAL = 1,        /* bad shape, dtype, pointer, alignment or workspace size    */
  XSAKE_EUNSUPPORTED = 2,  /* valid request outside what the kernels implement           */
  XSAKE_ECUDA = 3,         /* a CUDA runtime/driver call failed                          */
  XSAKE_ETIMEOUT = 4,      /* a bounded device-side wait gave up (see xsake_device_error) */
  XSAKE_EDEVICE = 5        /* a kernel recorded an error flag (see xsake_device_error)   */
};

enum { XSAKE_F32 = 0, XSAKE_BF16 = 1 };

/* ------------------------------------------------------------------ library status  */
XSAKE_API int xsake_abi_version(void);
XSAKE_API const char* xsake_last_error(void);
/* Reads and clears the device-side error word of the current device after
 * synchronising `stream`.  *code = 0 when no kernel recorded an error; otherwise a
 * packed (kind << 24 | detail) value.  Returns XSAKE_OK or XSAKE_ECUDA. */
XSAKE_API int xsake_device_error(void* stream, int32_t* code);

/* ------------------------------------------------------------------ block-mask plans
 * Replaces the per-call mask handling of the reference:
 *   _broadcast_mask                 kernels/pallas/sparse_attention.py:286-298
 *   token-mask expansion + causal   kernels/pallas/sparse_attention.py:76-81
 * A plan is compiled once per (mask, B, H, S, block_size, causal) and reused by every
 * attention call with that mask.  mask_dev is uint8 0/1 [mask_batch, mask_heads, nq, nk]
 * with mask_batch in {1, B}, mask_heads in {1, H}, nq = nk = S / block_size. */
typedef struct {
  int32_t batch, heads, seq;
  int32_t mask_batch, mask_heads;
  int32_t block_size;
  int32_t causal;
} XsakeMaskDims;

XSAKE_API int xsake_mask_plan_bytes(const XsakeMaskDims* dims, size_t* bytes);
XSAKE_API int xsake_mask_compile(const XsakeMaskDims* dims, const uint8_t* mask_dev, void* plan_dev,
                       size_t plan_bytes, void* stream);

/* Options of xsake_mask_compile_ex (the reference has no counterpart: it runs one job per device,
 * distributed/pmap_trainer.py:32-68).  units_dev (device memory, NULL = every unit) lists the
 * (b, h) units, as b * heads + h, that calls with this plan compute: a job whose batch x heads
 * is sharded over GPUs compiles on each rank a plan of its own units, and the attention calls
 * read and write only those units' rows of q, k, v, o, lse and the gradients.  workers is the
 * number of tile workers the forward runs concurrently (0 = 2 x the SM count of the current
 * device); the plan splits a query tile's kv walk into pieces when it is long next to the
 * average load of a worker, so a small job still fills the GPU.  Invalid unit ids are left out
 * and recorded in the device error word.  forward_pairing (one of XSAKE_PAIRING_*) fixes how the
 * tensor-core forward groups rows into work items; AUTO lets the plan compiler choose from the
 * mask, the others exist for measurement and tests (every pairing gives the same results up to
 * fp32 rounding of the softmax statistics). */
#define XSAKE_PAIRING_AUTO 0
#define XSAKE_PAIRING_QUERY 1   /* query chunks 2t, 2t+1 of one unit            */
#define XSAKE_PAIRING_UNITS 2   /* query chunk j of two units that share the mask */
typedef struct {
  const int32_t* units_dev;
  int32_t n_units;
  int32_t workers;
  int32_t forward_pairing;
} XsakePlanOptions;

XSAKE_API int xsake_mask_compile_ex(const XsakeMaskDims* dims, const XsakePlanOptions* options,
                       const uint8_t* mask_dev, void* plan_dev, size_t plan_bytes, void* stream);

/* Copies the plan's summary to host (synchronises `stream`): out[0] = active (q-block,
 * kv-block) pairs after the causal cut over the selected units, out[1] = 64x64 tiles the
 * forward computes with the pairing the plan chose, out[2] = fully masked q-blocks,
 * out[3] = forward work items. */
XSAKE_API int xsake_mask_plan_stats(const void* plan_dev, void* stream, int64_t out[4]);

/* The same summary and the plan compiler's choices (synchronises `stream`). */
typedef struct {
  int64_t active_blocks;    /* active (q-block, kv-block) pairs after the causal cut      */
  int64_t computed_tiles;   /* 64x64 tiles the tensor-core forward computes               */
  int64_t empty_qblocks;    /* fully masked q-blocks                                       */
  int32_t work_items;       /* forward work items, split pieces included                   */
  int32_t selected_units;   /* (b, h) units the plan computes                              */
  int32_t pairing;          /* forward pairing: 0 query chunks, 1 units                    */
  int32_t split_items;      /* work items cut into pieces over their kv chunks             */
  int32_t split_slots;      /* partial slots those pieces use                              */
  int32_t split_cap;        /* largest piece, in 64-key chunks                             */
  int32_t workers;          /* tile workers the split rule assumed                         */
  int32_t reserved;
} XsakePlanInfo;
XSAKE_API int xsake_mask_plan_info(const void* plan_dev, void* stream, XsakePlanInfo* info);

/* ------------------------------------------------------------------ attention
 * Replaces sparse_attention / sparse_attention_pallas / _sparse_attn_fwd_kernel
 * (kernels/pallas/sparse_attention.py:96-156, :161-252, :257-281) with the output
 * semantics of sparse_attention_reference (:45-91): token-level causal mask, and a fully
 * masked query row attends uniformly to all S keys (finfo.min fill).  lse[b,h,s] is the
 * natural-log row normaliser (finfo(float32).min for fully masked rows). */
typedef struct {
  int32_t dtype;            /* XSAKE_F32 or XSAKE_BF16 (q, k, v, o, do, dq, dk, dv)   */
  int32_t batch, heads, seq, head_dim;
  int32_t block_size;
  int32_t causal;
  int32_t mask_batch;       /* leading dims of the mask the plan was compiled from     */
  int32_t mask_heads;
  float scale;              /* softmax scale; <= 0 selects 1/sqrt(head_dim)           */
  int64_t q_stride[3];      /* element strides of (b, h, s); d stride is 1            */
  int64_t k_stride[3];
  int64_t v_stride[3];
  int64_t o_stride[3];      /* also used for do, dq, dk, dv                           */
} XsakeAttnDesc;

/* The forward's workspace (256-byte aligned) holds the work-item counter and, for the tensor-core
 * path, the partial results of split work items (about 17 MB); its first bytes are reset on the
 * stream by every call.  Only rows of the units the plan selects are written. */
XSAKE_API int xsake_attn_fwd_workspace_size(const XsakeAttnDesc* desc, size_t* bytes);
XSAKE_API int xsake_attn_fwd(const XsakeAttnDesc* desc, const void* plan_dev, const void* q_dev,
                   const void* k_dev, const void* v_dev, void* o_dev, float* lse_dev,
                   void* workspace_dev, size_t workspace_bytes, void* stream);

/* Backward of the above (the reference has no VJP; this is autodiff of
 * sparse_attention_reference, :45-91).  lse_dev is the forward's output.  The workspace must
 * be 256-byte aligned.  bf16 / head_dim 64 / block_size % 64 == 0 runs on the tensor cores
 * (deterministic: no atomics on the gradients); other configurations on CUDA cores. */
XSAKE_API int xsake_attn_bwd_workspace_size(const XsakeAttnDesc* desc, size_t* bytes);
XSAKE_API int xsake_attn_bwd(const XsakeAttnDesc* desc, const void* plan_dev, const void* q_dev,
                   const void* k_dev, const void* v_dev, const void* o_dev,
                   const float* lse_dev, const void* do_dev, void* dq_dev, void* dk_dev,
                   void* dv_dev, void* workspace_dev, size_t workspace_bytes, void* stream);

/* The attention weights, the second output of sparse_attention_reference (:45-91) that the
 * reference's calibration collects (training/trainer.py:79-117): p_dev (fp32, 16-byte aligned)
 * receives P[b, h, q, k] = softmax over all S keys of q.k * scale with masked entries at
 * finfo(float32).min, i.e. a fully masked row is uniform 1/S.  head_dim 32 or 64, fp32 or bf16
 * q/k through desc's strides; uses the plan's mask.  Scores are fp32-accurate: bf16 inputs at
 * head_dim 64 run on the tensor cores, everything else on the CUDA cores in fp32. */
XSAKE_API int xsake_attn_probs(const XsakeAttnDesc* desc, const void* plan_dev, const void* q_dev,
                   const void* k_dev, float* p_dev, void* stream);
/* The same weights with a caller workspace (xsake_attn_probs_workspace_size bytes, 256-byte
 * aligned), which lets fp32 inputs at head_dim 64 run on the tensor cores too (three bf16 parts
 * per operand, as xsake_entropy_qk).  No counterpart in the reference beyond the weights. */
XSAKE_API int xsake_attn_probs_workspace_size(const XsakeAttnDesc* desc, size_t* bytes);
XSAKE_API int xsake_attn_probs_ex(const XsakeAttnDesc* desc, const void* plan_dev, const void* q_dev,
                   const void* k_dev, float* p_dev, void* workspace_dev, size_t workspace_bytes,
                   void* stream);

/* compute_attention_entropy (kernels/hads/hads_pattern.py:36-50) of exactly the weights
 * xsake_attn_probs gives (masked by the plan, causal cut, finfo.min fill), without materialising
 * them: head_sums_dev[h] (fp64) = sum over (b, q) of -sum_k c log c, c = clip(p, 1e-9, 1).  This is
 * what the reference's calibration reduces (the layer-0 weights of training/trainer.py:79-117).
 * Strided q, k as in desc; the workspace is xsake_entropy_qk_workspace_size(batch, heads, seq)
 * bytes.  Deterministic. */
XSAKE_API int xsake_attn_entropy(const XsakeAttnDesc* desc, const void* plan_dev, const void* q_dev,
                   const void* k_dev, double* head_sums_dev, void* workspace_dev, size_t workspace_bytes,
                   void* stream);

/* ------------------------------------------------------------------ row kernels
 * fused_softmax / fused_softmax_pallas / _softmax_kernel
 * (kernels/pallas/fused_softmax.py:26-87): softmax over the last axis of a contiguous
 * [rows, cols] array, fp32 statistics, output in the input dtype. */
XSAKE_API int xsake_softmax_fwd(int32_t dtype, int64_t rows, int64_t cols, const void* x_dev,
                      void* y_dev, void* stream);
/* dx = y * (dy - sum(dy * y)) -- autodiff of the above. */
XSAKE_API int xsake_softmax_bwd(int32_t dtype, int64_t rows, int64_t cols, const void* y_dev,
                      const void* dy_dev, void* dx_dev, void* stream);

/* fused_layernorm / fused_layernorm_pallas / _layernorm_kernel
 * (kernels/pallas/fused_layernorm.py:26-119): x [rows, d] in x_dtype, gamma/beta fp32
 * [d], fp32 two-pass statistics, y in x_dtype.  mean_dev / rstd_dev may be NULL. */
XSAKE_API int xsake_layernorm_fwd(int32_t x_dtype, int64_t rows, int64_t d, const void* x_dev,
                        const float* gamma_dev, const float* beta_dev, float eps,
                        void* y_dev, float* mean_dev, float* rstd_dev, void* stream);
XSAKE_API int xsake_layernorm_bwd_workspace_size(int64_t rows, int64_t d, size_t* bytes);
/* dgamma / dbeta are fp32 [d] and are overwritten (deterministic column reduction). */
XSAKE_API int xsake_layernorm_bwd(int32_t x_dtype, int64_t rows, int64_t d, const void* x_dev,
                        const float* gamma_dev, const float* mean_dev, const float* rstd_dev,
                        const void* dy_dev, void* dx_dev, float* dgamma_dev, float* dbeta_dev,
                        void* workspace_dev, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------ cross entropy
 * cross_entropy_loss (model/transformer.py:177-203) of the config-4 training step, over
 * `rows` rows of logits (dtype XSAKE_F32 / XSAKE_BF16; the vocabulary is the last axis, ld
 * elements between rows, ld >= vocab).  targets_dev int64 [rows]; a target equal to
 * ignore_index contributes nothing (the reference's `valid` mask); other targets are clamped
 * to [0, vocab).  Forward: lse_dev[r] = log(sum exp logits[r]) and nll_dev[r] = lse - logit of
 * the target (0 when ignored), fp32 arithmetic; the caller sums nll and divides by the number
 * of valid rows.  Backward: grad_dev (same dtype and ld as the logits) receives
 * *coef_dev * (softmax - onehot(target)) in the vocab columns, 0 in columns [vocab, ld) and in
 * ignored rows; coef_dev is a device fp32 scalar (d loss / d sum of nll). */
XSAKE_API int xsake_xent_fwd(int32_t dtype, int64_t rows, int64_t vocab, int64_t ld, const void* logits_dev,
                   const int64_t* targets_dev, int64_t ignore_index, float* lse_dev, float* nll_dev,
                   void* stream);
XSAKE_API int xsake_xent_bwd(int32_t dtype, int64_t rows, int64_t vocab, int64_t ld, const void* logits_dev,
                   const int64_t* targets_dev, int64_t ignore_index, const float* lse_dev,
                   const float* coef_dev, void* grad_dev, void* stream);

/* ------------------------------------------------------------------ HADS calibration
 * compute_attention_entropy (kernels/hads/hads_pattern.py:36-50): p fp32
 * [B, H, Sq, Sk] contiguous; head_sums_dev[h] (fp64) receives sum over (b, q) of
 * -sum_k clip(p,1e-9,1) * log(clip(p,1e-9,1)).  The caller divides by B*Sq for the mean,
 * or all-reduces the sums across ranks first.  Deterministic (fixed reduction order). */
XSAKE_API int xsake_entropy_workspace_size(int64_t batch, int64_t heads, int64_t sq, size_t* bytes);
XSAKE_API int xsake_entropy_rows(const float* p_dev, int64_t batch, int64_t heads, int64_t sq,
                       int64_t sk, double* head_sums_dev, void* workspace_dev,
                       size_t workspace_bytes, void* stream);

/* compute_attention_entropy of softmax(Q K^T * scale) without materialising P: q, k contiguous
 * [B, H, S, D] (fp32 or bf16, D 32 or 64), no mask (the calibration pass attends fully,
 * hads_pattern.py:118-166 via training/trainer.py:79-117); scale <= 0 selects 1/sqrt(D).
 * head_sums_dev[h] = sum over (b, q) of the clipped row entropy, as xsake_entropy_rows gives for
 * the materialised P.  D = 64: tensor cores, an fp32 operand split into three bf16 parts whose
 * six leading products give fp32-accurate scores (bf16 inputs: one product); D = 32: fp32 on
 * the CUDA cores.  Deterministic.  The workspace (xsake_entropy_qk_workspace_size bytes, 256-byte
 * aligned) holds the per-tile partial sums and the bf16 parts of K (~3 * B * H * S * 128 bytes). */
XSAKE_API int xsake_entropy_qk_workspace_size(int64_t batch, int64_t heads, int64_t seq, size_t* bytes);
XSAKE_API int xsake_entropy_qk(int32_t dtype, const void* q_dev, const void* k_dev, int64_t batch,
                       int64_t heads, int64_t seq, int64_t head_dim, float scale,
                       double* head_sums_dev, void* workspace_dev, size_t workspace_bytes,
                       void* stream);

/* Same result as xsake_entropy_rows for callers that can neither pass a workspace nor allocate
 * device memory (a framework plugin that may only use its framework's allocator, a process
 * whose device memory is all held by a pool allocator, a loop that cannot afford cudaMalloc's
 * device synchronisation).  It has no counterpart in the reference: the reference never
 * manages device memory itself.  Scratch is a library-owned static device array of 65,536
 * fp64 partial sums (512 KiB on every GPU that loads the library): calls needing more
 * (batch * heads * ctas_per_slice, ctas_per_slice = seq_q / largest divisor of seq_q <= 16)
 * return XSAKE_EUNSUPPORTED.  The first call on a device resolves the array's address; make it
 * before any stream capture.  All calls share the array, so calls overlapping on the GPU race. */
XSAKE_API int xsake_entropy_rows_noalloc(const float* p_dev, int64_t batch, int64_t heads,
                       int64_t sq, int64_t sk, double* head_sums_dev, void* stream);

/* ------------------------------------------------------------------ calibration exchange
 * The single collective of the path: a float64 sum all-reduce of the per-head entropy sums
 * (xsake_entropy_rows output) across ranks, so every rank builds the same masks.  Replaces the
 * reference's cross-device reduction (jax.lax.pmean, distributed/pmap_trainer.py:54-55) for
 * calibration (training/trainer.py:79-117), for callers without torch.distributed.  NCCL is
 * loaded at run time (libnccl.so.2); without it these calls return XSAKE_EUNSUPPORTED.
 * Rank 0 calls xsake_comm_unique_id and hands the 128 bytes to every rank out of band; each
 * rank then calls xsake_comm_init with the CUDA device it will use current. */
XSAKE_API int xsake_comm_unique_id(uint8_t id_out[128]);
/* xsake_comm_init_ex with a 300 s bound. */
XSAKE_API int xsake_comm_init(const uint8_t id[128], int nranks, int rank, void** comm_out);
/* Failure handling (the reference has none on this path): the communicator is non-blocking and
 * every host-side wait of this rank is bounded by timeout_ms (<= 0: unbounded).  A rank that
 * never joins makes init return XSAKE_ETIMEOUT after timeout_ms, with the communicator aborted;
 * the process and its GPU stay usable. */
XSAKE_API int xsake_comm_init_ex(const uint8_t id[128], int nranks, int rank, int timeout_ms, void** comm_out);
/* In place on buf_dev (count doubles), stream-ordered on `stream`; returns once the collective is
 * enqueued (bounded by the communicator's timeout). */
XSAKE_API int xsake_comm_allreduce_sum_f64(void* comm, double* buf_dev, size_t count, void* stream);
/* Waits on the host, at most timeout_ms, until `stream` has finished the collectives enqueued on
 * it.  A peer that died or never entered the collective: the communicator is aborted (which ends
 * its kernels still waiting on the stream) and XSAKE_ETIMEOUT returned; destroy it afterwards. */
XSAKE_API int xsake_comm_wait(void* comm, void* stream, int timeout_ms);
XSAKE_API int xsake_comm_destroy(void* comm);

#ifdef __cplusplus
}
#endif

#endif /* XSAKE_HADS_H */
