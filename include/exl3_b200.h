/*
 * exl3_b200.h - C ABI of the B200-native EXL3 trellis-decode matmul library
 * (libexl3b200.so).
 *
 * Plain pointers and sizes only: every tensor argument is a device pointer, every
 * stream argument a cudaStream_t passed as void*.  Functions return 0 on success
 * or one of the EXL3B200_E* codes below; they never exit the process and never
 * allocate device memory: outputs and workspaces are the caller's.  All work is
 * enqueued on the given stream; nothing synchronises the host.
 *
 * Data formats are the reference's (vcruz305/sglang-exl3):
 *   trellis  int16 [k/16, n/16, 16*K]   16x16 tiles of K-bit trellis codes
 *            (src/sglang_exl3/dense.py:140-150, exl3.py:1987-2071)
 *   suh      fp16 [k]   input sign/scale,  svh fp16 [n]  output sign/scale
 *   K        bits per weight; cb codebook: 0 = 3INST, 1 = MCG, 2 = mul1
 *            (the reference's bool mcg maps to cb 1 / cb 2, dense.py:151-157)
 * The weight the codes stand for is W = diag(suh) H W_raw H diag(svh) / 128 with H
 * the 128-point Walsh-Hadamard matrix, and the matmul ops compute y = x @ W.
 */
#ifndef EXL3_B200_H
#define EXL3_B200_H

#include <stddef.h>

#if defined(__GNUC__)
#define EXL3B200_API __attribute__((visibility("default")))
#else
#define EXL3B200_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* status codes */
#define EXL3B200_OK 0
#define EXL3B200_EBADSHAPE 1
#define EXL3B200_EBADBITS 2
#define EXL3B200_EBADCODEBOOK 3
#define EXL3B200_EUNALIGNED 4
#define EXL3B200_ELAUNCH 5
#define EXL3B200_EWORKSPACE 6
#define EXL3B200_ENULL 7
#define EXL3B200_EBADARG 8
#define EXL3B200_ETIMEOUT 9
#define EXL3B200_EIO 10

/* output dtypes */
#define EXL3B200_DTYPE_F16 0
#define EXL3B200_DTYPE_BF16 1
#define EXL3B200_DTYPE_F32 2

/* flags of the matmul entry points */
#define EXL3B200_FLAG_INPUT_ROTATED 1 /* x is already H128(x*suh)/sqrt(128) in fp16; suh unused */
#define EXL3B200_FLAG_SINGLE_CTA 2    /* exl3b200_gemm: no CTA-pair tiles (otherwise from 2048 rows, k >= 16384) */
#define EXL3B200_FLAG_PAIR_CTA 4      /* exl3b200_gemm: CTA-pair tiles at any row count (n a multiple of 256) */

/* largest row count of the small-M matmul */
#define EXL3B200_GEMV_MAX_M 16
/* most linears in one exl3b200_gemv_multi call */
#define EXL3B200_MULTI_MAX 8

/* ABI version of this header (the reference exposes P2B_MOE_ABI_VERSION = 2,
 * csrc/bindings.cpp:170; this library's ABI is versioned separately) */
#define EXL3B200_ABI_VERSION 1

EXL3B200_API int exl3b200_abi_version(void);
EXL3B200_API const char* exl3b200_status_string(int status);

/*
 * Kernel-shape map: which kernel family serves a problem.  Replaces the
 * reference's select_gemm_shape / exl3_gemm_num_kernel_shapes /
 * exl3_gemm_shape_compat (csrc/quant/exl3_kernel_map.cuh:3-5), whose table of
 * mma.sync tile shapes lives in the unvendored exllamav3.  The B200 table is keyed
 * by rows (per problem, or per expert for routed MoE), K and the matrix size, from
 * crossovers measured on a B200 (the numbers are in the table's comments).
 * GV16 above 16 rows means 16-row chunks of the small-M kernel.
 */
#define EXL3B200_SHAPE_GV8 1       /* small-M, one 8-row group, 8 tiles per warp, 2 CTAs per SM */
#define EXL3B200_SHAPE_GV8_NARROW 2 /* small-M, one 8-row group, 4 tiles per warp, 3 CTAs per SM */
#define EXL3B200_SHAPE_GV16 3      /* small-M, two 8-row groups (9..16 rows) */
#define EXL3B200_SHAPE_TC 4        /* tcgen05, 256 x 256 tiles, persistent, whole tiles then stream-K */
#define EXL3B200_SHAPE_MOE_SMALL 5 /* routed MoE on the grouped small-M pipeline */
#define EXL3B200_SHAPE_MOE_TC 6    /* routed MoE on grouped tcgen05 GEMMs */

typedef struct exl3b200_shape_desc {
    const char* name;
    int max_rows;     /* rows one launch of this shape takes per problem (0 = any) */
    int tile_rows;    /* rows of one output tile (8, 16 or 256) */
    int tile_cols;    /* output columns of one tile (128 or 256) */
    int ctas_per_sm;
} exl3b200_shape_desc;

EXL3B200_API int exl3b200_num_shapes(void);
/* experts == 0: a dense matmul of m rows; experts > 0: a routed MoE layer of m tokens
 * with topk experts each over `experts` local experts.  Returns a shape id. */
EXL3B200_API int exl3b200_select_shape(int m, int k, int n, int K, int cb, int experts, int topk);
/* 1 when the shape can run the problem (rows, k/n multiples of 128, K 2..4), else 0 */
EXL3B200_API int exl3b200_shape_compat(int shape, int m, int k, int n, int K);
EXL3B200_API int exl3b200_shape_info(int shape, exl3b200_shape_desc* out);

/*
 * Reconstruct the fp16 weight W [k, n] (row-major) from its trellis.
 * Replaces sglang_exl3_c.dequant_trellis (reference csrc/bindings.cpp:117-132,
 * op signature src/sglang_exl3/ops.py:38-54).  k and n must be multiples of 128,
 * K in 1..8.  rounding 0: codebook rounded to nearest, as the reference's device
 * decode (csrc/quant/codebook.cuh); rounding 1: truncated, bit-identical to the
 * reference's CPU dequant_trellis output (csrc/exl3_dequant.cuh:41-93).
 */
EXL3B200_API int exl3b200_dequant(const void* trellis, int k_tiles, int n_tiles, int K, int cb,
                     const void* suh, const void* svh, void* out, int rounding, void* stream);

/*
 * Small-M matmul: out[m, n] = x[m, k] @ W for 1 <= m <= 16.
 * Replaces sglang_exl3_c.exl3_gemv (reference csrc/bindings.cpp:134-147,
 * csrc/exl3_gemv.cu:26-63; op src/sglang_exl3/ops.py:57-74) and the row chunks of
 * exl3_gemm (csrc/exl3_gemm.cu:9-31).  x fp16 with row stride x_stride elements;
 * out in out_dtype with row stride out_stride elements (so outputs can be written
 * into a slice of a wider buffer).  K in 2..4, k and n multiples of 128.
 *
 * state:   exl3b200_gemv_state_size(n) bytes, 256-byte aligned, ZEROED once when
 *          allocated; every call leaves it zeroed again.  Calls that may run
 *          concurrently (different streams) need distinct state buffers.
 * scratch: exl3b200_gemv_scratch_size(m, k) bytes, 256-byte aligned, no
 *          initialisation; also per concurrent stream.
 */
EXL3B200_API size_t exl3b200_gemv_state_size(int n);
EXL3B200_API size_t exl3b200_gemv_scratch_size(int m, int k);
EXL3B200_API int exl3b200_gemv(const void* x, long long x_stride, int m, int k, const void* trellis, int n, int K,
                  int cb, const void* suh, const void* svh, void* out, long long out_stride,
                  int out_dtype, int flags, void* state, size_t state_bytes, void* scratch,
                  size_t scratch_bytes, void* stream);

/*
 * Small-M matmul with a routed, weighted fp32 accumulation instead of a store:
 * out[out_rows[r], :] += (out_scale ? out_scale[r] : 1) * (x[r] @ W) for r < m.
 * out_rows (int32) and out_scale (fp32) are DEVICE arrays of m entries; rows of
 * one call must be distinct.  Replaces sglang_exl3_c.exl3_fat_gemm_scatter's
 * accumulation (reference csrc/exl3_fat_gemm.cu:177-190) for small row counts.
 * Workspaces as for exl3b200_gemv.
 */
EXL3B200_API int exl3b200_gemv_combine(const void* x, long long x_stride, int m, int k, const void* trellis, int n,
                                       int K, int cb, const void* suh, const void* svh, float* out,
                                       long long out_stride, const int* out_rows, const float* out_scale,
                                       int flags, void* state, size_t state_bytes, void* scratch,
                                       size_t scratch_bytes, void* stream);

/*
 * The same routed, weighted accumulation for any m on the tensor cores (codes
 * decoded once per 256 rows): out[out_rows[r], :] += out_scale[r] * (x[r] @ W).
 * out_rows / out_scale may be NULL (row r, weight 1); repeated rows add up (fp32
 * vector atomics).  Replaces sglang_exl3_c.exl3_fat_gemm_scatter (reference
 * csrc/exl3_fat_gemm.cu:286-305, one tile pass per 128 rows there).  out must be
 * 16-byte aligned with out_stride a multiple of 4; scratch:
 * exl3b200_gemm_combine_scratch_size(m, k, n) bytes, 256-byte aligned, no
 * initialisation (no state buffer).
 */
EXL3B200_API size_t exl3b200_gemm_combine_scratch_size(int m, int k, int n);
EXL3B200_API int exl3b200_gemm_combine(const void* x, long long x_stride, int m, int k, const void* trellis, int n,
                                       int K, int cb, const void* suh, const void* svh, float* out,
                                       long long out_stride, const int* out_rows, const float* out_scale,
                                       int flags, void* scratch, size_t scratch_bytes, void* stream);

/*
 * Small-M matmul that allocates nothing and takes no workspace: out = x @ W as
 * exl3b200_gemv, for callers that cannot allocate device memory (an
 * allocator-less runtime that owns all device memory up front, or a thread that
 * must not enter the CUDA allocator).  Its scratch is one device array inside
 * the library (about 4 MB, held by every GPU that loads the library until the
 * process exits).  Limits: m <= 16, k <= 32768, n <= 32768; larger sizes return
 * EXL3B200_EBADSHAPE.  All calls share that array: calls that overlap on the GPU
 * race, so serialise them.  The first call on a device looks the array up and,
 * under CUDA's lazy module loading (the default), is also what loads the
 * library's device code on that device and so reserves the array: make one
 * warm-up call on each device before entering code that must not allocate, and
 * before capturing a stream.  This entry point has no counterpart in the
 * reference.
 */
EXL3B200_API int exl3b200_gemv_noalloc(const void* x, long long x_stride, int m, int k, const void* trellis, int n,
                                       int K, int cb, const void* suh, const void* svh, void* out,
                                       long long out_stride, int out_dtype, void* stream);

/*
 * Several linears over one input in a single launch sequence: out_i = x @ W_i for
 * i < count (count <= EXL3B200_MULTI_MAX), all with the same K, codebook and k.
 * Replaces the upstream exllamav3 exl3_mgemm pair GEMM the reference calls for
 * merged gate_up / k,v projections (src/sglang_exl3/dense.py:91-119,345-357) and
 * serves fused q/k/v.  Arrays are host arrays of device pointers.  state:
 * sum over i of exl3b200_gemv_state_size(n[i]) bytes, zeroed once; scratch:
 * count * exl3b200_gemv_scratch_size(m, k) bytes.
 */
EXL3B200_API int exl3b200_gemv_multi(int count, const void* x, long long x_stride, int m, int k, int K, int cb,
                                     const void* const* trellis, const int* n, const void* const* suh,
                                     const void* const* svh, void* const* out, const long long* out_stride,
                                     int out_dtype, int flags, void* state, size_t state_bytes, void* scratch,
                                     size_t scratch_bytes, void* stream);

/*
 * Batched experts: out[e] = x_e @ W_{expert_ids[e]} for e < count, out laid out
 * [count][m][n] in out_dtype; x_e = x (x_per_expert 0) or x + e*m*x_stride.
 * trellis/suh/svh_ptrs are DEVICE int64 tables of device pointers indexed by
 * expert id (table_size entries); expert_ids is a DEVICE int32 list read on the
 * device (ids are clamped to the table).  Replaces sglang_exl3_c.p2b_gemv_batched
 * (reference csrc/p2b_batched.cu:13-101, op src/sglang_exl3/ops.py:96-118) for
 * any codebook.  state: exl3b200_batched_state_size bytes, zeroed once.
 */
EXL3B200_API size_t exl3b200_batched_state_size(int count, int m, int n);
EXL3B200_API size_t exl3b200_batched_scratch_size(int count, int m, int k);
EXL3B200_API int exl3b200_batched_gemv(const void* x, int x_per_expert, long long x_stride, int m, int k, int n,
                                       int K, int cb, const long long* trellis_ptrs, const long long* suh_ptrs,
                                       const long long* svh_ptrs, int table_size, const int* expert_ids, int count,
                                       void* out, int out_dtype, void* state, size_t state_bytes, void* scratch,
                                       size_t scratch_bytes, void* stream);

/*
 * Routed SwiGLU MoE for tokens <= max_tokens rows of x [tokens, hidden] (fp16):
 *   out[t] (+)= sum_j w[t,j] * down_e(silu(min(gate_e x_t, L)) * clamp(up_e x_t, -L, L)),
 *   e = topk_ids[t, j], w = topk_weights[t, j]; ids outside [0, num_experts) are
 *   skipped.  L = swiglu_limit (0 or infinite: no clip).  out is fp32 [tokens,
 *   out_stride]; it is zeroed first unless accumulate != 0 (use accumulate to add a
 *   shared expert with a second call).  All tables are DEVICE int64 arrays of
 *   device pointers [num_experts]; topk_ids (int32) and topk_weights (fp32) are
 *   DEVICE [tokens, topk].  No host synchronisation.  Replaces
 *   sglang_exl3_c.p2b_fused_moe (reference csrc/p2b_moe.cu:418-468, op
 *   src/sglang_exl3/ops.py:121-184; fixed there to one row, hidden 4096) and the
 *   per-token batched GEMV path (src/sglang_exl3/exl3.py:960-1110).
 *   max_tokens * topk <= 65536, num_experts <= 2048.
 */
EXL3B200_API size_t exl3b200_moe_state_size(int max_tokens, int topk, int hidden, int inter);
EXL3B200_API size_t exl3b200_moe_scratch_size(int max_tokens, int topk, int hidden, int inter);
EXL3B200_API int exl3b200_moe(const void* x, long long x_stride, int tokens, int hidden, int inter,
                              const int* topk_ids, const float* topk_weights, int topk, int num_experts,
                              const long long* gate_trellis, const long long* gate_suh, const long long* gate_svh,
                              const long long* up_trellis, const long long* up_suh, const long long* up_svh,
                              const long long* down_trellis, const long long* down_suh, const long long* down_svh,
                              int K_gate, int K_up, int K_down, int cb, float swiglu_limit, float* out,
                              long long out_stride, int accumulate, int max_tokens, void* state, size_t state_bytes,
                              void* scratch, size_t scratch_bytes, void* stream);

/*
 * The same routed SwiGLU MoE (same arguments and result) on the tensor cores, for
 * batches whose experts receive many rows each: every expert's codes are decoded
 * once per 256 of its rows into tcgen05 MMAs (exl3b200_moe streams them once per 16
 * rows).  Replaces the reference's large-M expert path, the per-expert loop over
 * sglang_exl3_c.exl3_fat_gemm / exl3_fat_gemm_scatter (src/sglang_exl3/exl3.py:
 * 1154-1231, csrc/exl3_fat_gemm.cu:65-305), without its host synchronisation.
 * scratch: exl3b200_moe_tc_scratch_size bytes, 256-byte aligned, no initialisation
 * (no state buffer).  out must be 16-byte aligned with out_stride a multiple of 4.
 * max_tokens * topk <= 65536, num_experts <= 2048.
 */
EXL3B200_API size_t exl3b200_moe_tc_scratch_size(int max_tokens, int topk, int num_experts, int hidden, int inter);
EXL3B200_API int exl3b200_moe_tc(const void* x, long long x_stride, int tokens, int hidden, int inter,
                                 const int* topk_ids, const float* topk_weights, int topk, int num_experts,
                                 const long long* gate_trellis, const long long* gate_suh, const long long* gate_svh,
                                 const long long* up_trellis, const long long* up_suh, const long long* up_svh,
                                 const long long* down_trellis, const long long* down_suh,
                                 const long long* down_svh, int K_gate, int K_up, int K_down, int cb,
                                 float swiglu_limit, float* out, long long out_stride, int accumulate,
                                 int max_tokens, void* scratch, size_t scratch_bytes, void* stream);

/*
 * out[m, k] = H128(x * suh) / sqrt(128) in fp16 over 128-element blocks of each row,
 * with the reference's roundings (fp16 product, float transform, one fp16
 * rounding: had_hf_r_128_inner<true,false>, csrc/quant/hadamard_inner.cuh:93-147).
 * suh may be NULL (no pre-scale).  Replaces the upstream exllamav3 had_r_128 that
 * the reference's fat-GEMM path calls (src/sglang_exl3/exl3.py:1184-1193).
 */
EXL3B200_API int exl3b200_hadamard_in(const void* x, long long x_stride, int m, int k, const void* suh,
                                      void* out, long long out_stride, void* stream);

/*
 * Large-M matmul on the tensor cores (tcgen05 MMA, TMEM accumulators):
 * out[m, n] = x[m, k] @ W for any m >= 1, one pass over the codes per 256 rows.
 * Replaces sglang_exl3_c.exl3_gemm for M > 8 (reference csrc/bindings.cpp:102-132,
 * csrc/exl3_gemm.cu:9-31; op src/sglang_exl3/ops.py:77-95) and the dense GEMM of
 * exl3_fat_gemm (csrc/exl3_fat_gemm.cu:65-305; pass EXL3B200_FLAG_INPUT_ROTATED and
 * an fp32 out).  K in 2..4, k and n multiples of 128, trellis 16-byte aligned.
 *
 * state:   exl3b200_gemm_state_size() bytes (a partial-sum slot per SM for the
 *          output tiles that two CTAs share), 16-byte aligned, ZEROED once when
 *          allocated; every call leaves it zeroed.  One per concurrent stream; it
 *          may be the same buffer as the small-M matmul's state on that stream.
 * scratch: exl3b200_gemm_scratch_size(m, k) bytes, 16-byte aligned, no
 *          initialisation, one per concurrently running stream (the rotated
 *          input, laid out as the tensor cores' shared-memory tiles).
 * svh must be 16-byte aligned.  A device-side wait that gives up (after 1 s)
 * ends the kernel early and records EXL3B200_ETIMEOUT in the library's device
 * status (exl3b200_device_status).
 */
EXL3B200_API size_t exl3b200_gemm_state_size(void);
EXL3B200_API size_t exl3b200_gemm_scratch_size(int m, int k);
EXL3B200_API int exl3b200_gemm(const void* x, long long x_stride, int m, int k, const void* trellis, int n, int K,
                               int cb, const void* suh, const void* svh, void* out, long long out_stride,
                               int out_dtype, int flags, void* state, size_t state_bytes, void* scratch,
                               size_t scratch_bytes, void* stream);

/*
 * Enqueue on stream a copy of the library's sticky device status (0 or the first
 * device-side error code, e.g. EXL3B200_ETIMEOUT) into *host_status, and reset it
 * when reset != 0.  *host_status is valid after the stream has synchronised.
 * No counterpart in the reference, whose kernels have no device-side waits.
 */
EXL3B200_API int exl3b200_device_status(int* host_status, int reset, void* stream);

/*
 * Limit, in nanoseconds of the GPU's global timer, of every bounded device-side wait
 * in kernels launched after this call (the tensor-core pipeline's barrier waits and
 * the decode peer exchange's arrival wait); 0 restores the defaults (1 s and 2 s).
 * Process-wide.  A short limit lets a test make a wait run out quickly.  No
 * counterpart in the reference, whose kernels have no bounded waits.
 */
EXL3B200_API int exl3b200_set_wait_limit(unsigned long long ns);

/*
 * One EXL3 linear as the decode-layer entry points take it.
 */
typedef struct exl3b200_linear {
    const void* trellis; /* int16 [k/16][n/16][16K], 4-byte aligned */
    const void* suh;     /* fp16 [k] */
    const void* svh;     /* fp16 [n] */
    int k, n;
} exl3b200_linear;

/*
 * Dense SwiGLU MLP block: out = down(silu(clip(gate(x))) * clip(up(x))), with the
 * activation fused into the gate|up matmul's epilogue, which writes the down
 * projection's rotated input directly; no [m, 2 * inter] intermediate.  gate_up is
 * one fused EXL3 linear of n = 2 * inter columns (gate, then up), the layout the
 * reference's fat GEMM takes (packed13, src/sglang_exl3/exl3.py:1199-1218, which
 * runs the activation in torch between exl3_fat_gemm and had_r_128).  Roundings as
 * the reference: fp32 gate/up, fp16 activation, then the down projection's input
 * transform.  swiglu_limit 0 or infinite = no clip (gate clipped above, up to
 * [-limit, limit], csrc/p2b_moe.cu:304-313).  Up to 16 rows on the small-M kernels,
 * more on the tensor cores (exl3b200_select_shape); the tensor-core path wants the
 * trellises and svh 16-byte aligned.  state (zeroed once, left zeroed) and scratch
 * (no initialisation): exl3b200_mlp_workspace bytes, 256-byte aligned.  No
 * counterpart op in the reference.
 */
typedef struct exl3b200_mlp_args {
    const void* x;            /* fp16 [m][hidden], row stride x_stride */
    long long x_stride;
    int m, hidden, inter;
    exl3b200_linear gate_up;  /* k = hidden, n = 2 * inter */
    int K_gate_up, cb_gate_up;
    exl3b200_linear down;     /* k = inter, n = hidden */
    int K_down, cb_down;
    float swiglu_limit;
    void* out;                /* [m][hidden] in out_dtype, row stride out_stride */
    long long out_stride;
    int out_dtype;
} exl3b200_mlp_args;

EXL3B200_API int exl3b200_mlp_workspace(int m, int hidden, int inter, int K_gate_up, int cb_gate_up,
                                        size_t* state_bytes, size_t* scratch_bytes);
EXL3B200_API int exl3b200_mlp(const exl3b200_mlp_args* args, void* state, size_t state_bytes, void* scratch,
                              size_t scratch_bytes, void* stream);

/*
 * Peer buffers for tensor parallelism without NCCL in the decode sub-layers: one per
 * rank, allocated by its owner (the only allocating calls of the library, made once
 * at setup), mapped into every other rank's process through its 64-byte CUDA IPC
 * handle.  Each rank's buffer receives every rank's fp32 partial of a sub-layer and
 * the flags that say it has arrived.
 */
typedef struct exl3b200_peers {
    void* buffers[8];   /* every rank's buffer as mapped in this process; [rank] = own */
    int world, rank;    /* world <= 8 */
    int max_rows;       /* capacity the buffers were sized for (exl3b200_peer_buffer_size) */
    int hidden;
} exl3b200_peers;

EXL3B200_API size_t exl3b200_peer_buffer_size(int max_rows, int hidden);
EXL3B200_API int exl3b200_peer_buffer_alloc(size_t bytes, void** ptr, void* ipc_handle);
EXL3B200_API int exl3b200_peer_buffer_open(const void* ipc_handle, void** ptr);
EXL3B200_API int exl3b200_peer_buffer_close(void* ptr);
EXL3B200_API int exl3b200_peer_buffer_free(void* ptr);
/*
 * Enqueue on stream the re-arming of this rank's own peer buffer (call epoch 0, no
 * arrivals, not poisoned, next generation: values written before the reset are
 * never taken for a later call).  Every rank resets its own buffer once, while no
 * exchange is in flight on any rank.
 */
EXL3B200_API int exl3b200_peer_reset(void* own_buffer, void* stream);

/*
 * Expert-parallel routed MoE with the dispatch and the combine done over NVLink peer
 * memory by this library's kernels (no NCCL, no host synchronisation; CUDA-graph
 * capturable).  W = peers->world ranks each own experts / W experts (rank r: global
 * experts [r E/W, (r+1) E/W)) and each holds its own tokens; topk_ids are GLOBAL ids
 * (ids outside [0, experts) are skipped).  A token row goes once to every rank that
 * owns one of its experts (with its ids rewritten to that rank's local ids), each
 * rank runs its local experts with the routed SwiGLU pipeline (path 0: small-M, 1:
 * tensor cores, -1: by exl3b200_select_shape), the weighted results go back to the
 * token's rank and out[t] (fp32) is their sum.  Replaces SGLang's standard
 * dispatcher around the reference's MoE method (src/sglang_exl3/exl3.py:2254-2313;
 * expert ownership as exl3.py:485-509, 2089-2110).  tables: host array of the 9
 * DEVICE int64 pointer tables of this rank's experts (gate_trellis, gate_suh,
 * gate_svh, up_*, down_*; as exl3b200_moe).  Peer buffers: exl3b200_peer_buffer_alloc /
 * _open with exl3b200_ep_buffer_size(world, max_tokens, topk, hidden) bytes;
 * peers->max_rows = max_tokens, peers->hidden = hidden.  x and out 16-byte aligned
 * (x_stride a multiple of 8, out_stride of 4).  Every rank makes the same sequence
 * of calls.  Waits are bounded (exl3b200_set_wait_limit, default 2 s); a wait that
 * runs out records EXL3B200_ETIMEOUT, poisons the rank's buffer (later calls return
 * zeros) until exl3b200_peer_reset on every rank (see the decode sub-layers).
 * state / scratch: exl3b200_ep_workspace bytes, 256-byte aligned; state zeroed once.
 */
typedef struct exl3b200_ep_args {
    const void* x;              /* fp16 [tokens][hidden] */
    long long x_stride;
    int tokens, max_tokens;     /* this rank's tokens, and the capacity the buffers were sized for */
    int hidden, inter;
    const int* topk_ids;        /* int32 [tokens][topk] global ids */
    const float* topk_weights;  /* fp32 [tokens][topk] */
    int topk, experts;          /* experts: global count, a multiple of world */
    const void* const* tables;  /* 9 device pointer tables of this rank's experts */
    int K_gate, K_up, K_down, cb;
    float swiglu_limit;
    float* out;                 /* fp32 [tokens][hidden] */
    long long out_stride;
    int path;
} exl3b200_ep_args;

EXL3B200_API size_t exl3b200_ep_buffer_size(int world, int max_tokens, int topk, int hidden);
EXL3B200_API int exl3b200_ep_workspace(const exl3b200_ep_args* args, const exl3b200_peers* peers,
                                       size_t* state_bytes, size_t* scratch_bytes);
EXL3B200_API int exl3b200_ep_moe(const exl3b200_ep_args* args, const exl3b200_peers* peers, void* state,
                                 size_t state_bytes, void* scratch, size_t scratch_bytes, void* stream);

/*
 * Fused decode sub-layers of a Llama-style decoder for batch <= 16 sequences,
 * head_dim 128, query heads per kv head <= 16.  No counterpart in the reference,
 * whose layers call SGLang's norm / attention / activation kernels around the
 * EXL3 ops (dense.py:317-371); each step follows the unfused model (RMSNorm,
 * RoPE rotate-half, softmax attention over the bf16 cache, SwiGLU, residual).
 *
 * State is the residual stream h (fp32 [batch][hidden], row stride h_stride) and
 * two alternating per-row sum-of-squares buffers: a sub-layer reads ss_in
 * (sum of h^2 per row, for its RMSNorm), zeroes ss_out and - when y_out is NULL -
 * adds its output into h and the new sum of squares into ss_out.  With y_out
 * (tensor parallelism) it stores its fp32 partial output in y_out instead; after
 * the all-reduce, exl3b200_residual_add(h, y, ss_out) completes the sub-layer.
 * With peers (non-NULL; y_out ignored) the sub-layer exchanges the partials itself
 * through the peer buffers (each fp32 value stored over NVLink together with the
 * call's tag in one 8-byte store; a warp waits, bounded - 2 s unless
 * exl3b200_set_wait_limit says otherwise - until every rank's values of its block
 * row carry the tag) and adds their sum into h; every rank must make the same
 * sequence of calls.  A wait that gives up records EXL3B200_ETIMEOUT in the device
 * status, leaves the call epoch as it is and poisons this rank's buffer (block rows
 * already complete may have been added into h: the step is lost); every later
 * exchange on it returns at once (recording EXL3B200_ETIMEOUT again) until
 * exl3b200_peer_reset.  The caller checks exl3b200_device_status and recovers by
 * draining every rank's stream, then exl3b200_peer_reset on every rank's own
 * buffer, with a host barrier before and after the resets.
 *
 * Attention: k_cache / v_cache are this layer's bf16 [batch][kv_heads][max_ctx][128];
 * *pos (device) is the new token's position, the cache holds 0..pos-1 and the
 * call appends position pos; inv_freq is fp32 [64] (RoPE, rotate-half).
 * MLP: swiglu_limit 0 or infinite = no clamp.
 * state (zeroed once, left zeroed) and scratch sizes: the *_workspace functions;
 * 256-byte aligned; per concurrently running stream.
 */
EXL3B200_API int exl3b200_decode_attention_workspace(int batch, int hidden, int q_heads, int kv_heads, int max_ctx,
                                                     size_t* state_bytes, size_t* scratch_bytes);
EXL3B200_API int exl3b200_decode_mlp_workspace(int batch, int hidden, int inter, size_t* state_bytes,
                                               size_t* scratch_bytes);
EXL3B200_API int exl3b200_decode_attention(int batch, int hidden, int q_heads, int kv_heads, int K, int cb, float* h,
                                           long long h_stride, const float* ss_in, float* ss_out,
                                           const void* norm_w, float eps, const exl3b200_linear* q,
                                           const exl3b200_linear* k, const exl3b200_linear* v,
                                           const exl3b200_linear* o, void* k_cache, void* v_cache, int max_ctx,
                                           const long long* pos, const float* inv_freq, float* y_out,
                                           long long y_stride, const exl3b200_peers* peers, void* state,
                                           size_t state_bytes, void* scratch, size_t scratch_bytes, void* stream);
/*
 * The same attention sub-layer for several rows per sequence (speculative verify:
 * the last accepted token and the draft tokens): rows r = rows_per_seq * s + j
 * (rows % rows_per_seq == 0, rows <= 16) are sequence s at position *pos + j.  The
 * caches hold rows / rows_per_seq sequences; the call appends positions *pos ..
 * *pos + rows_per_seq - 1 of each, and row j attends to positions 0 .. *pos + j
 * (causal among the new rows).  rows_per_seq = 1 is exl3b200_decode_attention.
 * Workspace: exl3b200_decode_attention_workspace(rows, ...).  Replaces the per-token
 * verify loop around the reference's EXL3 ops (src/sglang_exl3/exl3.py:932-956).
 */
EXL3B200_API int exl3b200_decode_attention_rows(int rows, int rows_per_seq, int hidden, int q_heads, int kv_heads,
                                                int K, int cb, float* h, long long h_stride, const float* ss_in,
                                                float* ss_out, const void* norm_w, float eps, const exl3b200_linear* q,
                                                const exl3b200_linear* k, const exl3b200_linear* v,
                                                const exl3b200_linear* o, void* k_cache, void* v_cache, int max_ctx,
                                                const long long* pos, const float* inv_freq, float* y_out,
                                                long long y_stride, const exl3b200_peers* peers, void* state,
                                                size_t state_bytes, void* scratch, size_t scratch_bytes, void* stream);
EXL3B200_API int exl3b200_decode_mlp(int batch, int hidden, int inter, int K, int cb, float* h, long long h_stride,
                                     const float* ss_in, float* ss_out, const void* norm_w, float eps,
                                     const exl3b200_linear* gate, const exl3b200_linear* up,
                                     const exl3b200_linear* down, float swiglu_limit, float* y_out,
                                     long long y_stride, const exl3b200_peers* peers, void* state,
                                     size_t state_bytes, void* scratch, size_t scratch_bytes, void* stream);
EXL3B200_API int exl3b200_residual_add(int batch, int hidden, float* h, long long h_stride, const float* y,
                                       long long y_stride, float* ss_out, void* stream);

/*
 * A whole decoder layer (the attention sub-layer, then the MLP sub-layer) with the
 * RMSNorm input stages folded into the residual epilogues: the attention's residual
 * epilogue writes the MLP's normalised, rotated gate/up inputs itself, and - when
 * next is not NULL - the MLP's residual epilogue writes the next layer's q/k/v
 * inputs, which the next call (same rows, shapes, state and scratch; input_ready 1)
 * takes instead of running its input stage.  A residual epilogue does not know the
 * row's new norm yet, so it writes fp16(h * w * c) with c = rsqrt(ss_old/hidden +
 * eps) / 16 (the row's factor before the add, with 16x headroom) and the consuming
 * epilogue (RoPE/KV, SwiGLU) multiplies its outputs by rsqrt(ss_new/hidden + eps) / c:
 * the same linear map, rounded at other points (within the unfused sub-layers' fp16
 * tolerance); a row whose norm grows more than ~10^4-fold across one sub-layer
 * would overflow the fp16 input.  Two kernels fewer per layer than the two sub-layer
 * calls.
 *
 * ss_a: the rows' sum of squares of h on entry, and of the new h on return; ss_b: a
 * second fp32 [rows] buffer used in between.  The first layer of a step passes
 * input_ready 0 (its input stage normalises h).  Single GPU, or tensor parallel with
 * peers (the all-reduce form has no residual epilogue to fold into).  Everything
 * else as exl3b200_decode_attention_rows and exl3b200_decode_mlp; workspace:
 * exl3b200_decode_layer_workspace (state zeroed once, left zeroed).
 */
typedef struct exl3b200_decode_layer {
    const void* attn_norm_w;  /* bf16 [hidden] */
    const exl3b200_linear* q;
    const exl3b200_linear* k;
    const exl3b200_linear* v;
    const exl3b200_linear* o;
    const void* mlp_norm_w;   /* bf16 [hidden] */
    const exl3b200_linear* gate;
    const exl3b200_linear* up;
    const exl3b200_linear* down;
} exl3b200_decode_layer;

EXL3B200_API int exl3b200_decode_layer_workspace(int rows, int hidden, int q_heads, int kv_heads, int inter,
                                                 int max_ctx, size_t* state_bytes, size_t* scratch_bytes);
EXL3B200_API int exl3b200_decode_layer_step(int rows, int rows_per_seq, int hidden, int q_heads, int kv_heads,
                                            int inter, int K, int cb, float* h, long long h_stride, float* ss_a,
                                            float* ss_b, float eps, const exl3b200_decode_layer* layer,
                                            const exl3b200_decode_layer* next, int input_ready, void* k_cache,
                                            void* v_cache, int max_ctx, const long long* pos, const float* inv_freq,
                                            float swiglu_limit, const exl3b200_peers* peers, void* state,
                                            size_t state_bytes, void* scratch, size_t scratch_bytes, void* stream);

/*
 * Checkpoint reader: copies count byte ranges of the open file fd (offsets[i],
 * sizes[i] bytes) to dst[i].  Replaces the pread() loop of the reference's
 * exl3_mmap load format (src/sglang_exl3/loader.py:121-168), which reads every
 * tensor into a fresh host buffer for SGLang to copy to the GPU afterwards.
 *
 * dst_on_device 1: dst are device pointers.  staging is the caller's PINNED host
 * buffer of staging_bytes, split into `threads` slots (each a multiple of 4 KB,
 * at least 4 KB, else EXL3B200_EWORKSPACE); `threads` reader threads pread()
 * chunks into their slots and enqueue the host-to-device copies on `stream`.
 * dst_on_device 0: dst are host pointers, read into directly by the threads;
 * no CUDA call is made and staging may be NULL.
 * drop_cache 1: each range read is dropped from the page cache (posix_fadvise).
 * threads in 1..64.  Unlike the compute entry points this call blocks: it
 * returns once every byte is in place (device copies complete).  A file that
 * ends inside a range returns EXL3B200_EIO.
 */
EXL3B200_API int exl3b200_read_ranges(int fd, const long long* offsets, const long long* sizes, void* const* dst,
                                      int count, int dst_on_device, void* staging, size_t staging_bytes,
                                      int threads, int drop_cache, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* EXL3_B200_H */
