/*
 * qi4_b200.h - C ABI of the B200 (sm_100a) W4G64 QuantLinear backend.
 *
 * The library replaces the GPU side of the reference project
 * ryanyue-16/qwen2-int4-systems (paths below are relative to its root):
 * the dispatch target of QuantLinear.forward (src/qwen_int4/linear.py:56-72)
 * and the Triton operators behind it (src/qwen_int4/triton_kernels.py).
 *
 * Checkpoint contract read unchanged (src/qwen_int4/linear.py:39-44,
 * src/qwen_int4/quantization.py:30-84,221-258):
 *   qweight  uint8  N*K/2 bytes, row-major [N, K/2]; element k of row n sits
 *                   in byte (n*K + k)/2, low nibble for even k; signed INT4.
 *   scales   fp16   [N, K/64], one scale per row and 64-wide K group.
 *   zeros    uint8  (N*(K/64)+1)/2 bytes; signed INT4 zero point of
 *                   (row n, group g) is nibble (n*G+g)&1 of byte (n*G+g)/2.
 *                   NULL means all zero points are 0 (symmetric RTN).
 *   W[n,k] = (code[n,k] - zero[n,k/64]) * scale[n,k/64]
 *
 * Conventions: every pointer is a device pointer borrowed from the caller;
 * `stream` is a cudaStream_t (NULL = legacy default stream); calls only
 * enqueue work and never synchronise. Return value 0 means success; a
 * negative QI4_ERR_* code means nothing was launched (argument errors) or the
 * launch failed; qi4_last_error() then gives a message. No C++ exception
 * crosses this boundary. Calls on distinct streams may run concurrently.
 */
#ifndef QI4_B200_H
#define QI4_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define QI4_API __attribute__((visibility("default")))
#else
#define QI4_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Element types of activations, bias and outputs. */
#define QI4_DTYPE_NONE (-1)
#define QI4_DTYPE_F16 0
#define QI4_DTYPE_BF16 1
#define QI4_DTYPE_F32 2

/* Status codes. */
#define QI4_OK 0
#define QI4_ERR_ARGUMENT (-1)  /* null pointer or non-positive size */
#define QI4_ERR_DTYPE (-2)     /* unsupported element type */
#define QI4_ERR_SHAPE (-3)     /* K not a multiple of 64, size limits */
#define QI4_ERR_ALIGNMENT (-4) /* pointer alignment the kernels need */
#define QI4_ERR_LAUNCH (-5)    /* CUDA launch / runtime error */
#define QI4_ERR_DEVICE (-6)    /* current device is not sm_100 */

/* Kernel choice for qi4_w4g64_linear_ex. */
#define QI4_ALGO_AUTO 0 /* GEMV for small M, tensor-core GEMM otherwise */
#define QI4_ALGO_GEMV 1     /* TMA-staged, tensor-pipe decode GEMV (M <= 16) */
#define QI4_ALGO_TC 2       /* tcgen05 dequant-GEMM with TMEM accumulators */
#define QI4_ALGO_GEMV_FMA 3 /* CUDA-core FP32-FMA decode GEMV (M <= 16) */

/*
 * out[M, N] = x[M, K] @ W^T (+ bias[N]), FP32 accumulation, bias added in
 * FP32, result cast to x's dtype - the semantics of torch_reference_linear
 * (src/qwen_int4/backends.py:73-98) and of linear_canonical_w4g64_triton
 * (src/qwen_int4/triton_kernels.py:206-268).
 *   x        [M, K] row-major, dtype x_dtype (F16, BF16 or F32), 16-byte aligned
 *   qweight  16-byte aligned; scales 2-byte aligned
 *   bias     [N] of bias_dtype (F16/BF16/F32) or NULL with QI4_DTYPE_NONE
 *   out      [M, N] row-major, same dtype as x
 * K must be a positive multiple of 64; M, N positive.
 */
QI4_API int qi4_w4g64_linear(const void* x, int x_dtype, int64_t M, int64_t K,
                     const uint8_t* qweight, const uint16_t* scales_f16,
                     const uint8_t* zeros, const void* bias, int bias_dtype,
                     void* out, int64_t N, void* stream);

/* Same as qi4_w4g64_linear with an explicit kernel choice (QI4_ALGO_*) and
 * programmatic dependent launch on (pdl=1) or off (pdl=0). */
QI4_API int qi4_w4g64_linear_ex(const void* x, int x_dtype, int64_t M, int64_t K,
                        const uint8_t* qweight, const uint16_t* scales_f16,
                        const uint8_t* zeros, const void* bias, int bias_dtype,
                        void* out, int64_t N, void* stream, int algo, int pdl);

/*
 * out[N, K] = FP32 dequantised weight, bit-exact with dequantize_groupwise
 * (src/qwen_int4/quantization.py:221-258) and
 * dequantize_canonical_w4g64_triton (src/qwen_int4/triton_kernels.py:149-203).
 * out must be 16-byte aligned.
 */
QI4_API int qi4_w4g64_dequant_f32(const uint8_t* qweight, const uint16_t* scales_f16,
                          const uint8_t* zeros, float* out, int64_t N,
                          int64_t K, void* stream);

/*
 * out[i] = signed INT4 element i of `packed` (even i from the low nibble),
 * for 0 <= i < elements <= 2 * bytes; matches unpack_int4 CANONICAL
 * (src/qwen_int4/quantization.py:53-84) and
 * unpack_canonical_signed_int4_triton (src/qwen_int4/triton_kernels.py:119-146).
 * elements == 0 is a no-op.
 */
QI4_API int qi4_w4_unpack(const uint8_t* packed, int8_t* out, int64_t elements,
                  void* stream);

/*
 * Allocation-free form of qi4_w4g64_linear for FP32 activations (the input
 * dtype of the model's down_proj): out[M, N] (FP32) = x[M, K] (FP32) @ W^T
 * (+ bias), on the tensor-core kernel. No counterpart in the reference: it
 * exists for callers that cannot allocate device memory while serving a
 * request - engines that budget all device memory up front, FFI hosts with
 * no CUDA allocator of their own, loops that must not enter an allocator.
 * The FP32 path needs scratch (bf16 hi/lo copies of x); here it is a fixed
 * 32 MiB array in the library's device memory, present on every GPU that
 * loads the library until the process exits, so M * K <= 8388608 (larger
 * inputs return QI4_ERR_SHAPE; use qi4_w4g64_linear). The first call on a
 * device looks up the array's address (cudaGetSymbolAddress); make that first
 * call before any stream capture. All calls share the one array: calls that
 * may run at the same time on the GPU (different streams without ordering)
 * race on it. Nothing is carried over between calls - each call writes every
 * scratch byte it reads. The array's address is cached per device for the
 * life of the process: after cudaDeviceReset on a device, do not call this
 * entry point on that device again.
 */
QI4_API int qi4_w4g64_linear_f32_noalloc(const float* x, int64_t M, int64_t K, const uint8_t* qweight,
                                         const uint16_t* scales_f16, const uint8_t* zeros,
                                         const void* bias, int bias_dtype, float* out, int64_t N,
                                         void* stream);

/* Several linears that share one activation block, in one launch: for
 * i < count (1..3), outs[i] = x @ W_i^T (+ biases[i]) with W_i given by
 * qweights[i] / scales_f16[i] / zeros[i] (same format and rules as
 * qi4_w4g64_linear; N = Ns[i], K common). The pointer arrays are HOST arrays
 * of device pointers; zeros and biases may be NULL arrays or hold NULL
 * entries; bias_dtype applies to every bias. For M <= 16 the matrices share
 * one GEMV launch (the activations are staged once and one dependent launch
 * replaces `count`, e.g. q/k/v or gate/up of a decoder layer); for larger M
 * it issues one tensor-core launch per matrix. Outputs equal those of
 * `count` separate qi4_w4g64_linear calls within the GEMV tolerance. No
 * reference counterpart: the reference calls each QuantLinear separately
 * (src/qwen_int4/model.py:71-73 q/k/v, model.py:134-135 gate/up). */
QI4_API int qi4_w4g64_linear_multi(const void* x, int x_dtype, int64_t M, int64_t K, int count,
                                   const uint8_t* const* qweights, const uint16_t* const* scales_f16,
                                   const uint8_t* const* zeros, const void* const* biases, int bias_dtype,
                                   void* const* outs, const int64_t* Ns, void* stream);

/* Fused gate/up projection + SwiGLU of a decoder MLP: out[M, N] (FP32) =
 * silu(g) * u with g = x @ W_gate^T and u = x @ W_up^T, each rounded to the
 * activation dtype first (the dtype QuantLinear returns) - the tensor the
 * reference MLP hands to down_proj (src/qwen_int4/model.py:133-135, which
 * computes F.silu(gate(x).float()) * up(x).float()). Both matrices are
 * canonical W4G64 with the same K and N; no bias. For M <= 16 one GEMV launch
 * owns the same output rows of both matrices; larger M runs both projections
 * on the tensor cores, then an elementwise kernel. No reference counterpart as
 * a single call. */
QI4_API int qi4_w4g64_gate_up_silu(const void* x, int x_dtype, int64_t M, int64_t K, const uint8_t* qweight_gate,
                                   const uint16_t* scales_gate_f16, const uint8_t* zeros_gate,
                                   const uint8_t* qweight_up, const uint16_t* scales_up_f16,
                                   const uint8_t* zeros_up, float* out, int64_t N, void* stream);

/*
 * Column-split MLP over the GPUs of one node, the gather fused into the
 * SwiGLU pass. Replaces, for a rank's share of gate/up (output features
 * [col0, col0 + N) of the MLP's intermediate), the fused call above followed
 * by an all-gather of the FP32 intermediate (reference
 * src/qwen_int4/model.py:133-135 run with gate/up split by output features
 * over `world` ranks): the values, the same as qi4_w4g64_gate_up_silu's
 * (the projections rounded to the activation dtype first, then silu(g) * u
 * in FP32), are stored at outs[p][m * ld + col0 + n] for EVERY rank p - this
 * rank's own buffer and its peers' (device pointers valid on this GPU, e.g.
 * from qi4_ipc_open) - as they are produced. When every store of the call is
 * done, slot `rank` of every rank's flag array (flags[p], world + 1
 * zero-initialised 32-bit words: world flags, then that rank's CTA counter)
 * receives `epoch` with a system-scope release store. A consumer runs
 * qi4_peer_flag_wait on its own flag array with the same epoch before it
 * reads its gathered buffer. Epochs increase by one per call (wrapping
 * comparison). The caller keeps calls apart: a rank must not store into a
 * peer's buffer while that peer still reads the previous call's contents
 * (a collective that every rank passes after consuming, e.g. the gather of
 * the down_proj output, does it). N may be 0 (the epoch is still published).
 * world <= 8. Only plain stores reach peer memory (no TMA, no multicast).
 * No reference counterpart as a single call.
 */
QI4_API int qi4_w4g64_gate_up_silu_scatter(const void* x, int x_dtype, int64_t M, int64_t K,
                                           const uint8_t* qweight_gate, const uint16_t* scales_gate_f16,
                                           const uint8_t* zeros_gate, const uint8_t* qweight_up,
                                           const uint16_t* scales_up_f16, const uint8_t* zeros_up, int64_t N,
                                           float* const* outs, int64_t ld, int64_t col0, uint32_t* const* flags,
                                           int world, int rank, uint32_t epoch, void* stream);

/* Waits on the GPU (one small kernel on `stream`) until flags[r] has
 * reached `epoch` for every r < world, polling with acquire loads. A wait
 * longer than limit_ns (1 us .. 10 s) gives up, records
 * QI4_DEVICE_WAIT_TIMEOUT for qi4_device_status and lets the stream go on.
 * No reference counterpart (the all-gather it completes is NCCL's there). */
QI4_API int qi4_peer_flag_wait(const uint32_t* flags, int world, uint32_t epoch, uint64_t limit_ns, void* stream);

/* Buffers shared between the processes of one node (CUDA IPC, plain
 * peer-to-peer mappings; no multicast objects): qi4_ipc_alloc allocates
 * `bytes` of zeroed device memory on the current device and writes its
 * 64-byte handle; another process opens it with qi4_ipc_open (a pointer valid
 * on that process's current device) and unmaps it with qi4_ipc_close; the
 * owner frees it with qi4_ipc_free. These allocate, map and synchronise. No
 * reference counterpart. */
QI4_API int qi4_ipc_alloc(size_t bytes, void** ptr, void* handle);
QI4_API int qi4_ipc_open(const void* handle, void** ptr);
QI4_API int qi4_ipc_close(void* ptr);
QI4_API int qi4_ipc_free(void* ptr);

/*
 * Persistent decode chain (M <= 8 tokens): a fixed sequence of W4G64 linear
 * stages in which stage s + 1 reads what stage s (or an earlier stage)
 * wrote, run as ONE cooperative launch with one CTA per SM. It replaces a
 * chain of per-linear launches at decode sizes - the reference model's
 * QuantLinear calls of one decoder layer, src/qwen_int4/model.py:71-73
 * (q/k/v), :122 (o_proj) and :133-135 (gate/up/down), each of which the
 * reference dispatches separately through src/qwen_int4/linear.py:56-72 -
 * with one weight stream that runs across stage boundaries; the math of a
 * stage waits for its input on a device-side counter (bounded wait).
 *
 * A stage is 1..3 matrices sharing the activations x [M, K] (a device pointer:
 * external input or another stage's output) with the semantics of
 * qi4_w4g64_linear per matrix: out[m] [M, N[m]] = x @ W_m^T (+ bias[m]), FP32
 * accumulation, cast to out_dtype. With flags = QI4_CHAIN_SWIGLU the stage
 * holds {gate, up} (same N, no bias) and writes out[0] [M, N] in FP32 =
 * silu(g) * u, g and u rounded to x_dtype first (the reference MLP's
 * F.silu(gate(x).float()) * up(x).float(), model.py:133-135).
 *
 * qi4_chain_create validates the stages, copies every weight matrix into a
 * prepacked tile-major layout owned by the chain (the checkpoint buffers
 * are read, never modified; the copy is as large as qweight + scales +
 * zeros), allocates the chain's counters and scratch with cudaMalloc, and
 * synchronises `stream` once. The chain keeps the x / bias / out pointers:
 * those buffers must stay allocated, and a run reads whatever x holds when
 * it executes. qi4_chain_run enqueues one run on `stream` (no host sync);
 * runs of one chain must not overlap on the GPU (use one stream). A wait that
 * times out records QI4_DEVICE_WAIT_TIMEOUT for qi4_device_status.
 * qi4_chain_info reports: [0] CTAs, [1] ring slots per CTA, [2] shared
 * memory bytes, [3] prepacked bytes streamed per run, [4] algorithmic bytes
 * per run (canonical formula), [5] stages. No reference counterpart.
 */
#define QI4_CHAIN_SWIGLU 1
typedef struct qi4_chain_stage {
  int32_t nmats;      /* 1..3 (2 for QI4_CHAIN_SWIGLU: gate, up) */
  int32_t flags;      /* 0 or QI4_CHAIN_SWIGLU */
  int64_t K;          /* shared in_features, a multiple of 64 */
  const void* x;      /* [M, K] device pointer, 16-byte aligned */
  int32_t x_dtype;    /* F16, BF16 or F32 */
  int32_t bias_dtype; /* dtype of the non-null biases */
  int32_t out_dtype;  /* F16, BF16 or F32 (ignored for SwiGLU: F32) */
  int32_t reserved;
  const uint8_t* qweight[3];
  const uint16_t* scales_f16[3];
  const uint8_t* zeros[3]; /* NULL: symmetric (all zero points 0) */
  const void* bias[3];     /* NULL: no bias */
  void* out[3];            /* [M, N[m]]; SwiGLU: out[0] only */
  int64_t N[3];
} qi4_chain_stage;
typedef struct qi4_chain qi4_chain;
QI4_API int qi4_chain_create(const qi4_chain_stage* stages, int n_stages, int64_t M, void* stream,
                             qi4_chain** chain);
QI4_API int qi4_chain_run(qi4_chain* chain, void* stream);
QI4_API int qi4_chain_info(const qi4_chain* chain, int64_t* info);
QI4_API int qi4_chain_destroy(qi4_chain* chain);

/*
 * Decode attention with in-place KV-cache append, one new token per sequence
 * (bf16 throughout). Replaces, at decode, the reference attention's RoPE of
 * the new query/key (src/qwen_int4/model.py:74-77), its cache growth by
 * torch.cat and head expansion by repeat_interleave (model.py:80-91) and its
 * masked scaled_dot_product_attention (model.py:107-118):
 *   q', k' = RoPE(q, k) with cos/sin rows (bf16 roundings of the reference's
 *            q*cos + rotate_half(q)*sin); no RoPE when cos = sin = NULL
 *   k_cache[b, kvh, L_b] = k', v_cache[b, kvh, L_b] = v   (L_b = lengths[b])
 *   out[b, h*D:(h+1)*D] = softmax(q'_h K^T * scale) V over keys 0..L_b of KV
 *            head h / (Hq / Hkv), keys with key_mask[b, j] == 0 excluded
 * q [B, Hq, D], k_new / v_new [B, Hkv, D] contiguous; cos / sin rows of D
 * elements, row positions[b] (or b when positions is NULL); the caches are
 * [B, Hkv, capacity, D] at the given batch / head strides (elements, multiples
 * of 8; 16-byte aligned); lengths [B] int32 and the optional key_mask
 * [B, mask_stride] uint8 are device arrays, so a captured graph advances with
 * them. head_dim 128, at most 8 query heads per KV head. A sequence with
 * L_b >= capacity gets a zero output and QI4_DEVICE_CACHE_FULL. lengths is
 * not modified. No reference counterpart as a single call.
 */
#define QI4_DEVICE_CACHE_FULL 2
QI4_API int qi4_gqa_decode_attention(const void* q, const void* k_new, const void* v_new, const void* cos,
                                     const void* sin, const int32_t* positions, void* k_cache, void* v_cache,
                                     int64_t cache_batch_stride, int64_t cache_head_stride, int64_t cache_capacity,
                                     const int32_t* lengths, const uint8_t* key_mask, int64_t mask_stride,
                                     void* out, int64_t B, int64_t Hq, int64_t Hkv, int64_t head_dim, float scale,
                                     void* stream);

/* The same with a caller-owned workspace (`workspace_bytes` >= the size
 * qi4_gqa_decode_attention_workspace returns, 16-byte aligned; NULL: the
 * library's scratch pool), so that a captured graph holds only the kernels,
 * and flags: QI4_ATTN_EARLY_CACHE_READ lets the kernel read lengths,
 * positions and the past cache rows before it waits for the launch just
 * before it (it still waits before reading q, k_new and v_new) - only for
 * callers whose immediately preceding launches write none of them (a decode
 * step whose attention follows the q/k/v projection). cos / sin must be
 * 16-byte aligned. */
#define QI4_ATTN_EARLY_CACHE_READ 1
QI4_API size_t qi4_gqa_decode_attention_workspace(int64_t B, int64_t Hq, int64_t Hkv, int64_t cache_capacity);
QI4_API int qi4_gqa_decode_attention_ex(const void* q, const void* k_new, const void* v_new, const void* cos,
                                        const void* sin, const int32_t* positions, void* k_cache, void* v_cache,
                                        int64_t cache_batch_stride, int64_t cache_head_stride,
                                        int64_t cache_capacity, const int32_t* lengths, const uint8_t* key_mask,
                                        int64_t mask_stride, void* out, int64_t B, int64_t Hq, int64_t Hkv,
                                        int64_t head_dim, float scale, int flags, void* workspace,
                                        size_t workspace_bytes, void* stream);

/* Residual add + RMSNorm at a decoder block boundary (the reference's
 * DecoderLayer / RMSNorm, src/qwen_int4/model.py:31-42,151-159), in place on
 * the bf16 residual stream h [B, D]:
 *   h   = bf16(h + bf16(delta))   (delta [B, D] of BF16 or F32; NULL: none)
 *   out = bf16(bf16(h * rsqrt(mean(h^2) + eps)) * weight)   (FP32 statistics)
 * D <= 4096. No reference counterpart as a single call. */
QI4_API int qi4_add_rmsnorm(void* h, const void* delta, int delta_dtype, const void* weight, void* out, int64_t B,
                            int64_t D, float eps, void* stream);

/* The same block boundary folded into the next linear's activation staging
 * (decode sizes, bf16): the launch forms x = bf16(bf16(hn * rsqrt(mean(hn^2)
 * + eps)) * weight) from hn = bf16(h_in + bf16(delta)) itself, one launch
 * fewer per boundary, and writes hn to h_out. h_out must not overlap h_in
 * (callers alternate two residual buffers). */
typedef struct qi4_rmsnorm_prologue {
  const void* h_in;     /* bf16 [M, K] residual stream in */
  const void* delta;    /* BF16 or F32 [M, K] block output added to it, or NULL */
  int32_t delta_dtype;  /* QI4_DTYPE_BF16 or QI4_DTYPE_F32 */
  float eps;
  const void* weight;   /* bf16 [K] RMSNorm weight */
  void* h_out;          /* bf16 [M, K] residual stream out */
} qi4_rmsnorm_prologue;

/* qi4_w4g64_linear_multi with x formed by `norm` (bf16; 1 <= M <= 16; all
 * pointers of `norm` 16-byte aligned). */
QI4_API int qi4_w4g64_linear_multi_norm(const qi4_rmsnorm_prologue* norm, int64_t M, int64_t K, int count,
                                        const uint8_t* const* qweights, const uint16_t* const* scales_f16,
                                        const uint8_t* const* zeros, const void* const* biases, int bias_dtype,
                                        void* const* outs, const int64_t* Ns, void* stream);

/* qi4_w4g64_gate_up_silu with x formed by `norm` (same conditions). */
QI4_API int qi4_w4g64_gate_up_silu_norm(const qi4_rmsnorm_prologue* norm, int64_t M, int64_t K,
                                        const uint8_t* qweight_gate, const uint16_t* scales_gate_f16,
                                        const uint8_t* zeros_gate, const uint8_t* qweight_up,
                                        const uint16_t* scales_up_f16, const uint8_t* zeros_up, float* out,
                                        int64_t N, void* stream);

/*
 * Tied bf16 lm_head for decode sizes: logits[M, N] = x[M, K] @ W[N, K]^T
 * (bf16 in, FP32 sums, bf16 out - the reference's nn.Linear lm_head over the
 * tied embedding, src/qwen_int4/model.py:217-218,243) and/or argmax[M]
 * (int64) = the greedy token per row, taken over the bf16 logits with the
 * first index winning ties (generation.py:51, logits.argmax(dim=-1)).
 * Either output may be NULL (not both): a caller that needs only the greedy
 * token skips writing the logits. 1 <= M <= 8, K a multiple of 8 (<= 16384),
 * weight and x 16-byte aligned. No reference counterpart as a single call.
 */
QI4_API int qi4_bf16_gemv_argmax(const void* weight, const void* x, int64_t M, int64_t K, int64_t N, void* logits,
                                 int64_t* argmax, void* stream);

/* The same with a caller-owned argmax workspace: `keys` holds 8 64-bit words
 * that are zero on entry and left zero on return (the call's last kernel
 * resets them), so a captured graph needs no allocation or memset around it. */
QI4_API int qi4_bf16_gemv_argmax_ws(const void* weight, const void* x, int64_t M, int64_t K, int64_t N, void* logits,
                                    int64_t* argmax, uint64_t* keys, void* stream);

/* Greedy pick over bf16 logits rows, for batches the lm_head GEMV does not
 * take (the tied lm_head is then a library bf16 GEMM into `logits`): out[b] =
 * torch.argmax(logits[b, :V]) - the first index of the largest value, a NaN
 * counting as larger than every number. Rows are `ld` elements apart (ld >=
 * V). One CTA per row, programmatic dependent launch. Replaces the greedy
 * pick of reference src/qwen_int4/generation.py:51 (logits[:, -1].argmax).
 * Returns QI4_ERR_SHAPE unless 1 <= B < 2^31, 1 <= V < 2^32, ld >= V. */
QI4_API int qi4_bf16_argmax_rows(const void* logits, int64_t B, int64_t V, int64_t ld, int64_t* out, void* stream);

/* Tuning hook: forces the TMA/tensor-pipe GEMV launch shape for subsequent
 * calls made by the calling thread - output rows per CTA (16, 32, 64 or 128),
 * K-split factor (CTAs per cluster, 1..8) and warps per CTA (2, 4, 8, 16 or
 * 32, at least rows / 16). rows = 0 restores the library's own choice. No reference
 * counterpart. */
QI4_API int qi4_gemv_mma_plan_override(int rows, int ksplit, int warps);

/* Tuning hook: forces the tensor-core GEMM (M > 16) launch shape for
 * subsequent calls made by the calling thread - tokens per tile (32, 64, 128,
 * 192 or 256; FP32 activations at most 128) and the K split over a cluster
 * (1..8; above 1 only for tiles of at most 128 tokens). bn = 0 restores the
 * library's own choice. No reference counterpart. */
QI4_API int qi4_gemm_tc_plan_override(int bn, int ksplit);

/* Reports, without touching a GPU, the TMA/tensor-pipe GEMV launch plan the
 * library would use for an M x K activation block, N output features and
 * `num_sms` SMs: plan[0..5] = rows per CTA, K-split factor, warps per CTA,
 * 128-byte K boxes per CTA, dynamic shared memory in bytes, and 1 when the
 * weight fragments are expanded before the dependency wait. Returns QI4_OK,
 * or QI4_ERR_SHAPE when no plan exists (M outside 1..16 or K not a multiple of
 * 64). Honours qi4_gemv_mma_plan_override. No reference counterpart. */
QI4_API int qi4_gemv_mma_plan(int64_t M, int64_t N, int64_t K, int x_dtype, int num_sms, int64_t* plan);

/* Reads and clears the device-side error flags of the kernels (a bounded
 * wait that timed out records QI4_DEVICE_WAIT_TIMEOUT). Synchronises
 * `stream`. Returns the flags (0 = none) or a negative QI4_ERR_* code.
 * No reference counterpart (the reference has no device-side waits). */
#define QI4_DEVICE_WAIT_TIMEOUT 1
QI4_API int qi4_device_status(void* stream);

/* Failure-detection self-test: enqueues on `stream` one CTA that waits, with
 * the same bounded wait the kernels use, on a shared-memory barrier nothing
 * arrives on. The wait gives up after limit_ns (1 us .. 1 s) and records
 * QI4_DEVICE_WAIT_TIMEOUT, which the next qi4_device_status reports; the CUDA
 * context stays usable. Lets an operator check that a lost arrival ends as an
 * error status rather than a hang. No reference counterpart. */
QI4_API int qi4_selftest_bounded_wait(uint64_t limit_ns, void* stream);

/* Tuning hook: forces the FP32-FMA decode-GEMV launch shape for subsequent calls made
 * by the calling thread - lanes per weight row (8/16/32), warps per CTA,
 * K-split factor (CTAs per cluster, 1..8) and per-lane load depth (4 or 8).
 * lanes_per_row = 0 restores the library's own choice. No reference
 * counterpart (the reference's Triton tile is a wrapper argument,
 * src/qwen_int4/triton_kernels.py:213-216). */
QI4_API int qi4_gemv_plan_override(int lanes_per_row, int warps, int ksplit, int depth);

/* Copies the calling thread's last error message (NUL-terminated, truncated
 * to len) and returns its full length; 0 if no error was recorded. */
QI4_API int qi4_last_error(char* buf, size_t len);

/* ABI version of this header (major * 100 + minor). */
QI4_API int qi4_version(void);

#ifdef __cplusplus
}
#endif

#endif /* QI4_B200_H */
