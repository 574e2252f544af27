/*
 * dirktensor_b200 -- C ABI of the B200 (sm_100a) attention hot path.
 *
 * Drop-in boundary for DirkTensor's attention layer.  Each entry point names
 * the reference interface it replaces (file:line in the DirkTensor tree).
 * Plain pointers and sizes only; no C++ or torch types cross this boundary.
 * Nothing throws: every call returns a status code (DT_OK == 0) and
 * dt_last_error() gives a message for the calling thread.
 *
 * Layouts (as in the reference):
 *   activations  [B, T, H, D] or [B, T, d_model] row-major fp32 (d_model = H*D)
 *   weights      [out, in] row-major fp32 (the .npy checkpoint layout)
 *   statistics   softmax_m / softmax_l [B, T, H] fp32
 * Device-pointer entry points run asynchronously on `stream` (a cudaStream_t,
 * NULL = legacy default stream); *_host entry points take host buffers, copy
 * them to the device, run, copy back and synchronise.
 */
#ifndef DIRKTENSOR_B200_H
#define DIRKTENSOR_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status ------------------------------------------------------------ */
enum dt_status {
    DT_OK = 0,
    DT_ERR_INVALID_ARGUMENT = 1, /* bad shape, null or misaligned pointer        */
    DT_ERR_CUDA = 2,             /* a CUDA runtime/driver call failed            */
    DT_ERR_DEVICE_TIMEOUT = 3,   /* a kernel's bounded wait expired (no hang)    */
    DT_ERR_UNSUPPORTED = 4,      /* e.g. head_dim != 128, no sm_100 device       */
    DT_ERR_OUT_OF_MEMORY = 5,
    DT_ERR_IO = 6,               /* checkpoint file missing or malformed         */
    DT_ERR_NCCL = 7,             /* NCCL missing, or a communicator call failed  */
    DT_ERR_TIMEOUT = 8           /* a host-side wait (communicator set-up) expired */
};

/* Message for the last failing call on this thread ("" if none).
 * Replaces the reference's exceptions (std::runtime_error, xt::load_npy throws;
 * main.cpp:40, Detokenizer.cpp:44). */
const char* dt_last_error(void);

/* ABI version of this library (major * 10000 + minor * 100 + patch). */
int dt_version(void);

/* Synchronises the current device, then reports (and clears) a device-side
 * error recorded by a kernel whose bounded wait expired: DT_ERR_DEVICE_TIMEOUT.
 * The device-pointer entry points do not synchronise; call this after them. */
int dt_check_device_error(void);

/* Exercises the failure path on the current device: runs a kernel whose
 * barrier wait can never complete; the wait's 1-second budget expires, the
 * kernel records it and returns, and this call checks that the expiry was
 * reported (then clears it).  DT_OK means the mechanism works and the context
 * is still usable.  Takes about one second. */
int dt_selftest_expired_wait(void);

/* ---- flash attention forward -------------------------------------------
 * Replaces flash_attention_forward (FlashAttention.h:15-21,
 * FlashAttention.cpp:24-182) and fills FlashAttentionResult
 * (FlashAttention.h:6-10): o = softmax(scale * q k^T [+ causal mask]) v,
 * softmax_m = row max of the scaled scores, softmax_l = sum exp(s - m).
 * q, k, v, o: [B, T, H, D] fp32 device pointers; softmax_m/l may be NULL.
 * D must be 128.  Operands are rounded to bf16 for the tensor cores
 * (fp32 accumulation and softmax); the workspace holds the bf16 copies of K
 * and V (its first third, sized for Q, is unused: the attention kernel rounds
 * the rows of Q itself). */
size_t dt_flash_fwd_workspace_bytes(int B, int T, int H, int D);
int dt_flash_fwd(const float* q, const float* k, const float* v, float* o, float* softmax_m, float* softmax_l,
                 int B, int T, int H, int D, float scale, int causal, void* workspace, size_t workspace_bytes,
                 void* stream);
/* Same with host buffers (the call the C++ drop-in flash_attention_forward makes). */
int dt_flash_fwd_host(const float* q, const float* k, const float* v, float* o, float* softmax_m,
                      float* softmax_l, int B, int T, int H, int D, float scale, int causal);

/* Replaces flash_attention_backward (FlashAttention.h:33-43,
 * FlashAttention.cpp:185-359): from the upstream gradient dout, the forward
 * output out and statistics softmax_m / softmax_l (as dt_flash_fwd writes
 * them), and q, k, v, computes dq, dk, dv ([B,T,H,D] fp32 device arrays).
 * Operands are rounded to bf16 for the tensor cores; D = rowsum(out*dout) and
 * the softmax recomputation are fp32.  workspace: >= dt_flash_bwd_workspace_bytes,
 * 16-byte aligned.  Asynchronous on `stream`. */
size_t dt_flash_bwd_workspace_bytes(int B, int T, int H, int D);
int dt_flash_bwd(const float* dout, const float* out, const float* softmax_m, const float* softmax_l,
                 const float* q, const float* k, const float* v, float* dq, float* dk, float* dv, int B, int T,
                 int H, int D, float scale, int causal, void* workspace, size_t workspace_bytes, void* stream);
/* Same with host buffers (the call the C++ drop-in flash_attention_backward makes). */
int dt_flash_bwd_host(const float* dout, const float* out, const float* softmax_m, const float* softmax_l,
                      const float* q, const float* k, const float* v, float* dq, float* dk, float* dv, int B, int T,
                      int H, int D, float scale, int causal);

/* Same as dt_flash_fwd, but allocates nothing and takes no workspace: the
 * bf16 copies of K and V live in a fixed 24 MiB array inside the library's
 * device image (present on every GPU that loads the library until exit); Q is
 * rounded inside the attention kernel, so results are bit-identical to
 * dt_flash_fwd's.  No counterpart in the reference: it exists for callers that
 * cannot allocate device memory (an engine that owns its whole HBM budget
 * through its own pool, a plugin barred from allocating in callbacks, a loop
 * that cannot afford cudaMalloc's synchronisation).  B*T*H*D must be
 * <= 6,291,456, else DT_ERR_INVALID_ARGUMENT.  All calls share the array:
 * calls that may overlap on the GPU race and must be ordered by the caller.
 * The first call on a device looks up the array's address and caches it; make
 * it before any stream capture, and do not call again after cudaDeviceReset. */
int dt_flash_fwd_noalloc(const float* q, const float* k, const float* v, float* o, float* softmax_m,
                         float* softmax_l, int B, int T, int H, int D, float scale, int causal, void* stream);

/* Barrier of the in-kernel exchange (no counterpart in the reference, whose
 * heads share one process): after dt_flash_fwd_*_exchange on every rank, each
 * rank publishes `epoch` (a per-step counter starting at 1) into every rank's
 * flag array and waits, on the GPU, until every rank's epoch has arrived in its
 * own.  flag_bufs[r]: rank r's array of 8 uint32 (zero-initialised device
 * memory, mapped into this process, e.g. with dt_ipc_open; flag_bufs[rank] is
 * this rank's own).  The wait gives up after 1 second and records
 * DT_ERR_DEVICE_TIMEOUT (see dt_check_device_error).  Asynchronous on `stream`;
 * the O projection that reads the receive buffer goes after it. */
int dt_exchange_barrier(void* const* flag_bufs, int ranks, int rank, unsigned epoch, void* stream);

/* Packed-operand form used inside the layer and by head-sharded callers:
 * q, k, v are bf16 [B, T, H, D] device arrays; o is fp32 (o_bf16 = 0) or
 * bf16 (o_bf16 = 1) with o_row_stride elements between consecutive tokens
 * (H*D for the dense layout).  seq_lens (device int[B], may be NULL) gives
 * right-padded sequence lengths: rows t >= seq_lens[b] are written as zeros. */
int dt_flash_fwd_bf16(const void* q, const void* k, const void* v, void* o, int o_bf16, long long o_row_stride,
                      float* softmax_m, float* softmax_l, const int* seq_lens, int B, int T, int H, int D,
                      float scale, int causal, void* stream);

/* Flash attention fused with the head-parallel exchange (the head-sharded
 * form of flash_attention_forward + the reshape feeding OlmoAttention.cpp:99-107):
 * this rank (`rank` of `ranks`, <= 8) holds H heads of q, k, v (bf16
 * [B, T, H, D]); each output row of global token g = b*T + t is stored, bf16,
 * straight into recv_bufs[g / tokens_per_rank] -- this GPU's own receive buffer
 * or a peer's, mapped with dt_ipc_open -- at plane `rank`, row
 * g % tokens_per_rank.  A receive buffer is [ranks][tokens_per_rank][H*D]
 * bf16, the planar A operand of dt_gemm_bf16_tn_planar.  Two launches on
 * `stream`: the attention kernel, then a one-thread system-scope fence that
 * makes its peer stores visible system-wide.  The caller orders the owners'
 * reads after every rank's launches (e.g. a one-element all-reduce on the
 * same stream) and double-buffers the receive buffers across steps. */
int dt_flash_fwd_bf16_exchange(const void* q, const void* k, const void* v, void* const* recv_bufs, int ranks,
                               int rank, long long tokens_per_rank, float* softmax_m, float* softmax_l, int B, int T,
                               int H, int D, float scale, int causal, void* stream);

/* Same as dt_flash_fwd_bf16 and dt_flash_fwd_bf16_exchange, with Q given as fp32
 * [B, T, H, D] (K and V bf16): the attention kernel reads the fp32 rows of Q
 * and rounds them to bf16 itself, so no separate cast pass over Q is needed.
 * Results are identical to casting Q with dt_cast_f32_bf16 first. */
int dt_flash_fwd_qf32(const float* q, const void* k, const void* v, void* o, int o_bf16, long long o_row_stride,
                      float* softmax_m, float* softmax_l, const int* seq_lens, int B, int T, int H, int D,
                      float scale, int causal, void* stream);
int dt_flash_fwd_qf32_exchange(const float* q, const void* k, const void* v, void* const* recv_bufs, int ranks,
                               int rank, long long tokens_per_rank, float* softmax_m, float* softmax_l, int B, int T,
                               int H, int D, float scale, int causal, void* stream);
/* CUDA IPC for the exchange buffers.  dt_ipc_get_handle writes the 64-byte
 * handle of the allocation holding dev_ptr and dev_ptr's offset inside it;
 * dt_ipc_open maps a peer's handle (peer access enabled lazily) and returns the
 * mapped base + offset; dt_ipc_close unmaps it (same pointer and offset). */
int dt_ipc_get_handle(const void* dev_ptr, void* handle_out, size_t* offset_out);
int dt_ipc_open(const void* handle, size_t offset, void** dev_ptr_out);
int dt_ipc_close(void* dev_ptr, size_t offset);

/* ---- attention layer ----------------------------------------------------
 * Replaces class OlmoAttention (OlmoAttention.h:10-42): constructor
 * (OlmoAttention.cpp:39-53) and forward (OlmoAttention.cpp:56-108):
 *   y = (flash(rope(qnorm(x Wq^T)), rope(knorm(x Wk^T)), x Wv^T)) Wo^T
 * with RMSNorm over all d_model columns (RMSNorm.cpp:15-22), rotate-half RoPE
 * (OlmoAttention.cpp:18-36,111-146) and scale 1/sqrt(head_dim). */
typedef struct dt_attn dt_attn;

typedef struct dt_attn_weights {
    const float* q_proj; /* [d_model, d_model] host fp32, [out, in] */
    const float* k_proj;
    const float* v_proj;
    const float* o_proj;
    const float* q_norm; /* [d_model] */
    const float* k_norm;
    int d_model;         /* 2048 (model_config.h:5) */
    int n_heads;         /* 16   (model_config.h:6); head_dim must be 128 */
    float eps;           /* RMSNorm eps, 1e-6 (RMSNorm.h:10) */
    float rope_theta;    /* 500000 (OlmoAttention.cpp:16) */
} dt_attn_weights;

/* Uploads the weights (bf16 copies for the tensor cores) to `device`. */
int dt_attn_create(const dt_attn_weights* w, int device, dt_attn** out);
/* Reads {folder}/model.layers.{index}.self_attn.{q,k,v,o}_proj.weight.npy and
 * {q,k}_norm.weight.npy (float32, C order), as OlmoAttention.cpp:39-46 does. */
int dt_attn_create_from_npy(const char* folder, unsigned index, int device, dt_attn** out);
/* x, y: [B, T, d_model] fp32 device pointers.  seq_lens: device int[B] or
 * NULL; with it, rows t >= seq_lens[b] of y are zero (right padding). */
int dt_attn_forward(dt_attn* attn, const float* x, int B, int T, const int* seq_lens, float* y, void* stream);
/* Same with host buffers; seq_lens is a host int[B] or NULL. */
int dt_attn_forward_host(dt_attn* attn, const float* x, int B, int T, const int* seq_lens, float* y);
/* Training path of the layer (OlmoAttention::backward / step / zero_grad,
 * OlmoAttention.cpp:189-330, RMSNorm.cpp:24-41).  dt_attn_backward takes the
 * gradient dy of the last dt_attn_forward's output (same B, T; that forward
 * without seq_lens), writes dx (fp32 [B, T, d_model] device array) and adds the
 * weight gradients into the handle's fp32 gradient buffers (Wq, Wk, Wv, Wo,
 * q_norm, k_norm), which start at zero and are cleared by dt_attn_zero_grad.
 * dt_attn_step applies w -= lr * grad to the fp32 master weights (kept on the
 * device since creation) and refreshes the bf16 copies the kernels read.
 * dt_attn_get_params_host copies the weights (gradients = 0) or the gradients
 * (gradients = 1) to host arrays (nulls skipped), after a device sync. */
int dt_attn_backward(dt_attn* attn, const float* dy, int B, int T, float* dx, void* stream);
int dt_attn_backward_host(dt_attn* attn, const float* dy, int B, int T, float* dx);
int dt_attn_step(dt_attn* attn, float lr, void* stream);
int dt_attn_zero_grad(dt_attn* attn, void* stream);
int dt_attn_get_params_host(dt_attn* attn, float* q_proj, float* k_proj, float* v_proj, float* o_proj, float* q_norm,
                            float* k_norm, int gradients);
int dt_attn_destroy(dt_attn* attn);

/* ---- head-parallel attention layer (several GPUs of one node) ------------
 * The reference runs every head of a layer in one process, parallelising the
 * attention core over batch x heads (FlashAttention.cpp:43-45).  Here the 16
 * heads are split over G = 1, 2, 4 or 8 GPUs, one process (or thread) per GPU:
 * rank r owns heads [r*16/G, (r+1)*16/G).  Per forward, on every rank:
 *   [q|k|v]_r = x [Wq_r; Wk_r; Wv_r]^T        (rows of this rank's heads only)
 *   s_r = per-token sums of squares of q_r, k_r; all-reduce over the ranks
 *         (QK-RMSNorm normalises over all 2048 columns, RMSNorm.cpp:17, so it
 *         needs every rank's heads: 2 floats per token cross NVLink)
 *   q_r, k_r = RoPE(q_r / rms * g), v_r          (this rank's heads)
 *   attention on this rank's heads; each output row is stored into the rank
 *         that owns its token (token slice [r*M/G, (r+1)*M/G), M = B*T) --
 *         by the attention kernel itself over NVLink (exchange 0) or by an
 *         NCCL all-to-all (exchange 1)
 *   y_r = A_r Wo^T for this rank's token slice, A_r = all heads of its tokens.
 * x is the full [B, T, d_model] input on every rank; y is this rank's token
 * slice [B*T/G, d_model] (rows r*M/G ... of the flattened [B*T, d_model]).
 *
 * Communicator: one NCCL communicator per rank, created from a 128-byte id
 * that rank 0 makes with dt_comm_unique_id and hands to the other ranks
 * (files, sockets, MPI -- the library does not care).  dt_comm_create
 * initialises it without blocking and gives up after timeout_ms (aborting the
 * half-built communicator) with DT_ERR_TIMEOUT, so a rank that never joins
 * cannot hang the others' set-up.  NCCL is loaded at run time (libnccl.so.2);
 * without it these calls return DT_ERR_NCCL and nothing else is affected. */
typedef struct dt_comm dt_comm;
int dt_comm_unique_id(void* id_out /* 128 bytes */);
int dt_comm_create(const void* id, int world, int rank, int device, int timeout_ms, dt_comm** out);
/* Aborts the communicator's outstanding work (for a caller's watchdog). */
int dt_comm_abort(dt_comm* comm);
int dt_comm_destroy(dt_comm* comm);
/* Uploads this rank's share of the layer (its heads' rows of Wq, Wk, Wv, all
 * of Wo and of the norm gains) to the communicator's device.  Every rank
 * passes the same full weights.  exchange: 0 = attention kernel stores into
 * the owners' buffers over NVLink (CUDA IPC; all ranks on one node), 1 = NCCL
 * all-to-all.  Collective: every rank calls it. */
int dt_attn_create_sharded(const dt_attn_weights* w, dt_comm* comm, int exchange, dt_attn** out);
/* Collective forward (every rank, same B, T, seq_lens, gather).  x:
 * [B, T, d_model] fp32 device array (the full input).  gather = 0: y is this
 * rank's token slice [B*T/G, d_model]; gather = 1: y is the whole output
 * [B, T, d_model] on every rank (the token slices all-gathered in place, what
 * a caller that adds the residual, as OlmoBlock.cpp:14-16 does, needs).  B*T
 * must be divisible by G.  seq_lens: device int[B] or NULL (right padding:
 * rows t >= seq_lens[b] of y are zero).  Enqueued on `stream`; the NCCL calls
 * use the same stream.  The handle is destroyed with dt_attn_destroy; the
 * communicator outlives it. */
int dt_attn_forward_sharded(dt_attn* attn, const float* x, int B, int T, const int* seq_lens, int gather, float* y,
                            void* stream);
/* Same with host buffers (x: [B, T, d_model]; y: the slice or, with gather,
 * the whole output; seq_lens: host int[B] or NULL): copies in, runs the
 * collective forward on the handle's own stream, copies out, synchronises. */
int dt_attn_forward_sharded_host(dt_attn* attn, const float* x, int B, int T, const int* seq_lens, int gather,
                                 float* y);
/* dt_attn_create_sharded with the weights read from the checkpoint files of
 * layer `index` in `folder`, as dt_attn_create_from_npy reads them. */
int dt_attn_create_sharded_from_npy(const char* folder, unsigned index, dt_comm* comm, int exchange, dt_attn** out);

/* ---- full model prefill (configuration 3) -------------------------------
 * Replaces OlmoModel::forward (OlmoModel.cpp:25-48) with OlmoBlock::forward
 * (OlmoBlock.cpp:13-21), OlmoMlp::forward (OlmoMlp.cpp:26-63) and
 * OlmoLmHead::forward (OlmoLmHead.cpp:11-28): x = embed[ids]; per layer
 * h = x + RMSNorm(attn(x)), x = h + RMSNorm(mlp(h)); logits = RMSNorm(x) Wlm^T.
 * The residual stream stays fp32; GEMM operands are bf16 copies. */
typedef struct dt_model dt_model;

typedef struct dt_model_layer_weights {
    const float* q_proj; /* [d, d] */
    const float* k_proj;
    const float* v_proj;
    const float* o_proj;
    const float* q_norm; /* [d] */
    const float* k_norm;
    const float* post_attention_norm;   /* [d] */
    const float* gate_proj;             /* [hidden, d] */
    const float* up_proj;               /* [hidden, d] */
    const float* down_proj;             /* [d, hidden] */
    const float* post_feedforward_norm; /* [d] */
} dt_model_layer_weights;

typedef struct dt_model_weights {
    const float* embed;      /* [vocab, d] */
    const float* final_norm; /* [d] */
    const float* lm_head;    /* [vocab, d] */
    const dt_model_layer_weights* layers;
    int n_layers;            /* 16 (model_config.h:7) */
    int vocab;               /* 100352; multiple of 8 */
    int d_model;             /* 2048 */
    int n_heads;             /* 16 */
    int hidden;              /* 8192; multiple of 128 */
    float eps;
    float rope_theta;
} dt_model_weights;

int dt_model_create(const dt_model_weights* w, int device, dt_model** out);
/* Reads the checkpoint folder as OlmoModel.cpp:11-22 does (n_layers <= 0 means 16). */
int dt_model_create_from_npy(const char* folder, int n_layers, int device, dt_model** out);
/* tokens: uint32 [B, T] device; logits: fp32 [B, T, vocab] device.  Token ids
 * must be below vocab (the gather clamps, it does not check). */
int dt_model_forward(dt_model* m, const uint32_t* tokens, int B, int T, float* logits, void* stream);
/* Host buffers; token ids are checked against the vocabulary. */
int dt_model_forward_host(dt_model* m, const uint32_t* tokens, int B, int T, float* logits);
int dt_model_destroy(dt_model* m);
/* Layer count, vocabulary and MLP width of a created model (any may be NULL). */
int dt_model_info(const dt_model* m, int* n_layers, int* vocab, int* hidden);

/* ---- stages (for stage-wise parity checks and head-sharded callers) ----- */
/* dst[i] = bf16(src[i]), n elements (n % 4 == 0). */
int dt_cast_f32_bf16(const float* src, void* dst, long long n, void* stream);
/* dst0 = bf16(src0) and dst1 = bf16(src1), n elements each (n % 4 == 0), in one
 * launch (the K and V operands of the head-parallel attention step). */
int dt_cast2_f32_bf16(const float* src0, const float* src1, void* dst0, void* dst1, long long n, void* stream);
/* C[M,N] = A[M,K] . B[N,K]^T; A, B bf16 row-major device; C fp32 (c_bf16 = 0)
 * or bf16 (c_bf16 = 1) with ldc elements per row.  K % 8 == 0.
 * The projection products of OlmoAttention.cpp:68,74,80,103-105. */
int dt_gemm_bf16_tn(const void* A, const void* B, void* C, int c_bf16, int M, int N, int K, long long ldc,
                    void* stream);
/* General form: C (+)= op(A) . op(B)^T with bf16 operands.  a_mn = 0: A is
 * [M, K] row-major; a_mn = 1: A is stored [K, M] row-major (the transposed
 * operand).  b_mn = 0: B is [N, K]; b_mn = 1: B is stored [K, N].  c_mode: 0
 * store fp32, 1 store bf16, 2 add into an fp32 C.  Replaces the training
 * path's sgemm calls: dW += dY^T X (OlmoAttention.cpp:201-205, 250-267; a_mn =
 * b_mn = 1, c_mode = 2) and dX = dY W (:207, 278-298; b_mn = 1).  An MN-major
 * operand needs its M (or N) to be a multiple of 8. */
int dt_gemm_bf16(const void* A, int a_mn, const void* B, int b_mn, void* C, int c_mode, int M, int N, int K,
                 long long ldc, void* stream);
/* The same product with a planar A: a_planes arrays [M, K/a_planes] stored
 * back to back (A[m, p*(K/a_planes) + x] = plane_p[m, x]); K/a_planes must be a
 * multiple of 64.  This is the O projection (OlmoAttention.cpp:103-105) of the
 * head-parallel path: after the all-to-all, plane p holds source rank p's heads
 * for this rank's token slice. */
int dt_gemm_bf16_tn_planar(const void* A, int a_planes, const void* B, void* C, int c_bf16, int M, int N, int K,
                           long long ldc, void* stream);
/* Prologue: per token row r (position r % T), q/k RMSNorm over d_model = 2048
 * with gains, rotate-half RoPE (head_dim 128), v copied; outputs bf16
 * [B*T, 2048].  q, k, v: fp32 device rows with ld_in elements per row. */
int dt_qk_norm_rope(const float* q, const float* k, const float* v, long long ld_in, const float* q_gain,
                    const float* k_gain, void* q_out, void* k_out, void* v_out, int B, int T, float eps,
                    float rope_theta, void* stream);
/* Head-sharded prologue, first step: ss[r] = {sum q^2, sum k^2} over the
 * `width` columns of row r of q and k (fp32, ld elements per row; width a
 * multiple of 4).  Summed over the ranks, these are the full-row sums. */
int dt_qk_sumsq(const float* q, const float* k, long long ld, int width, long long M, float* ss, void* stream);
/* Head-sharded prologue, second step, for `heads` (1, 2, 4, 8, 16) heads:
 * q, k normalised with the full-row sums ss ([M, 2] fp32) and this rank's
 * slice of the gains (q_gain, k_gain: [heads*128]), RoPE'd; v copied; outputs
 * bf16 [M, heads*128] with M = B*T. */
int dt_qk_norm_rope_shard(const float* q, const float* k, const float* v, long long ld_in, const float* ss,
                          const float* q_gain, const float* k_gain, int heads, void* q_out, void* k_out, void* v_out,
                          int B, int T, float eps, float rope_theta, void* stream);
/* Host copy of the RoPE tables the device uses ([max_seq, head_dim] each),
 * computed like compute_rope_buffers (OlmoAttention.cpp:18-36). */
int dt_rope_tables(float* sin_out, float* cos_out, int max_seq, int head_dim, float theta);

#ifdef __cplusplus
}
#endif

#endif /* DIRKTENSOR_B200_H */
