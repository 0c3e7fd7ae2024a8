// Fused decode layer around the EXL3 small-M matmul: the glue of a Llama-style
// decoder layer (RMSNorm, RoPE, KV-cache append, attention, residual adds,
// SwiGLU) moved into the matmul pipeline's own input stages and epilogues, so a
// decode step runs ten kernels per layer instead of ~75 (eight with the norm fold).
//
// Attention sub-layer (exl3b200_decode_attention), all launches chained by
// programmatic dependent launch:
//   1. input stage, norm mode: x = fp16(h * rsqrt(ss/hidden + eps) * w) (ss = the
//      row's sum of squares, accumulated by the previous residual epilogue), then
//      the usual fp16 x*suh, H128, /sqrt(128) for each of q, k, v; zeroes the
//      sum-of-squares buffer the next residual epilogue accumulates into;
//   2. grouped matmul over q, k, v;
//   3. epilogue, RoPE/KV mode: each (row, head) block of q and k is rotated
//      (rotate-half pairs (d, d+64) sit in one lane of the warp-wide H128 layout),
//      q is stored scaled by 1/sqrt(head_dim), k and v are appended to the bf16
//      cache at the current position - with one row per sequence and every
//      cluster resident at once, done by the attention kernel's own warps (its
//      cluster's blocks) instead of a kernel;
//   4. split-K attention on the tensor cores: one thread-block cluster of up to
//      16 CTAs per (row, kv head); each CTA takes every 16th 64-position chunk
//      through a three-buffer cp.async ring whose first fill is requested before
//      the dependency wait (only q and the new row come from step 3), four warps
//      of 16 positions each.  The query heads of the GQA group (up to 16,
//      zero-padded) are the M rows of mma.m16n8k16 (bf16, fp32 accumulate; q and
//      the softmax weights enter as bf16 hi + lo pairs, two MMAs each): S = Q K^T,
//      a running softmax per warp, then P V with the score accumulators reused as
//      the A fragments.  The CTAs exchange their partials (unnormalised O, max,
//      sum) through distributed shared memory; rank r merges heads r, r + 16, ...
//      (log-sum-exp rescale), normalises, rounds to fp16 and writes the o
//      projection's rotated input (x*suh, H128);
//   5. matmul (o);
//   6. epilogue, residual mode: h += y and the row's new sum of squares (or, with
//      tensor parallelism, an fp32 store of the partial y for the all-reduce).
// MLP sub-layer (exl3b200_decode_mlp): norm input stage for gate and up, their
// grouped matmul, the SwiGLU epilogue that writes the down projection's rotated
// input, the down matmul and the residual epilogue.
//
// Tensor parallelism without NCCL (peers != NULL): the o / down matmul's epilogue
// kernel does the exchange itself - each warp stores its block row's fp32 partials,
// each with the call's tag in one 8-byte store, into its slot of every rank's peer
// buffer (CUDA IPC mapping, plain stores over NVLink), reads every rank's slots of
// the same block row from its own buffer until they carry the tag (bounded, 2 s),
// then adds their sum into h and accumulates the sum of squares.  Slots alternate
// between two parities by call.
//
// Whole layers (exl3b200_decode_layer_step) fold the RMSNorm input stages into the
// residual epilogues: the attention's residual epilogue writes the MLP's gate/up
// inputs and the MLP's writes the next layer's q/k/v inputs, pre-scaled by the row's
// norm factor before the add; the RoPE and SwiGLU epilogues multiply by the ratio of
// the exact factor to it.  Eight kernels per layer instead of ten.
//
// The reference has no decode-layer fusion (its layers call SGLang's norm,
// attention and activation kernels around the EXL3 ops); the arithmetic of each
// step follows the unfused model in exl3_b200/harness.py.
#include <algorithm>
#include <climits>
#include <cstring>

#include <cooperative_groups.h>

#include "exl3_common.cuh"
#include "exl3_capi_internal.h"
#include "exl3_grouped.cuh"
#include "exl3_grouped_dev.cuh"
#include "exl3_epilogue.cuh"

namespace exl3b200 {

namespace cg = cooperative_groups;

constexpr int kDecChunk = 64;   // attention positions per CTA

__global__ __launch_bounds__(256) void exl3_dec_input_kernel(const __grid_constant__ GvArgs a,
                                                             const __grid_constant__ DecAux x)
{
    griddep_launch();
    const int lane = threadIdx.x & 31;
    {
        // before the wait: the first task's norm weights and input scales into L2
        const int task = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
        if (task < a.in_tasks) {
            const GvProblem& p = gv_prob(a, gv_find<0>(a, a.nprob, task));
            const int b = (task - p.in_task_begin) % (p.k >> 7);
            prefetch_l2_256(x.norm_w + b * 128, lane);
            if (p.suh) prefetch_l2_256(p.suh + b * 128, lane);
        }
    }
    griddep_wait();
    if (x.ss_out && blockIdx.x == 0)
        for (int i = threadIdx.x; i < x.zero_rows; i += blockDim.x) x.ss_out[i] = 0.f;
    const int warps = gridDim.x * (blockDim.x >> 5);
    for (int task = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); task < a.in_tasks; task += warps) {
        const int pi = gv_find<0>(a, a.nprob, task);
        const GvProblem& p = gv_prob(a, pi);
        const int nblk = p.k >> 7;
        const int local = task - p.in_task_begin;
        const int r = local / nblk;
        const int b = local - r * nblk;
        float xv[4];
        {
            const float rs = rsqrtf(x.ss_in[r] * x.inv_hidden + x.eps);
            const float* hr = x.h + (size_t) r * x.h_stride + b * 128;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int c = lane + 32 * i;
                xv[i] = __half2float(__float2half_rn(hr[c] * rs * __bfloat162float(x.norm_w[b * 128 + c])));
            }
        }
        store_rotated(p.xd, p.sblk, p.suh, p.k, r, b, lane, xv);
    }
}

// Decode epilogues (RoPE/KV, SwiGLU, residual).  With the norm fold the RoPE and
// SwiGLU epilogues take over the skipped input stage's duty of zeroing the sum of
// squares that the sub-layer's residual epilogue accumulates (zero_ss).
template <int CB, int MODE>
__global__ __launch_bounds__(256) void exl3_dec_epilogue_kernel(const __grid_constant__ GvArgs a,
                                                                const __grid_constant__ DecAux x)
{
    griddep_launch();
    const int lane = threadIdx.x & 31;
    gv_prefetch_epilogue(a, lane);
    if (MODE == kEpiResidual && x.fold_n) {
        const int task = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
        if (task < a.out_tasks) fold_prefetch(x, task % (gv_prob(a, 0).n >> 7), lane);
    }
    griddep_wait();
    if (x.zero_ss && blockIdx.x == 0)
        for (int i = threadIdx.x; i < x.zero_rows; i += blockDim.x) x.zero_ss[i] = 0.f;
    const int warps = gridDim.x * (blockDim.x >> 5);
    for (int task = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); task < a.out_tasks; task += warps) {
        const int pi = gv_find<1>(a, a.nprob, task);
        const GvProblem& p = gv_prob(a, pi);
        const int nblocks = p.n >> 7;
        const int local = task - p.out_task_begin;
        const int r = local / nblocks;
        const int nb = local - r * nblocks;
        if constexpr (MODE == kEpiSwiglu) {
            // (gate, up) = table entries j and j + 1 (a stride-2 view of the table)
            const GvProblem& pu = a.inl[pi * a.stride + a.offset + 1];
            epi_block_row<CB>(a, x, MODE, pi, p, &pu, nb, r, lane);
        } else {
            epi_block_row<CB>(a, x, MODE, pi, p, nullptr, nb, r, lane);
        }
    }
}

// ---------------------------------------------------------------------------
// split-K decode attention on the tensor cores: one thread-block cluster per
// (row, kv head), partials merged through distributed shared memory
// ---------------------------------------------------------------------------

constexpr int kAttnWarps = kDecChunk / 16;  // 16 positions of a chunk per warp
constexpr int kAttnThreads = 32 * kAttnWarps;
constexpr int kAttnMaxGroup = 16;           // query heads per kv head (the M rows of the MMA)
constexpr int kAttnMaxCluster = 16;         // CTAs per (row, kv head)
constexpr int kKvPitch = kHeadDim + 8;      // bf16 per staged K/V row: 272 B, ldmatrix rows on distinct banks
constexpr int kOPitch = kHeadDim + 8;       // fp32 per row of a warp's partial O

constexpr int kAttnBufs = 3;                // K/V chunk ring; all three requested before the dependency wait

struct AttnSmem {
    union {
        __nv_bfloat16 kv[kAttnBufs][2][kDecChunk][kKvPitch];  // [buffer][K, V][position][dim]
        float o[kAttnWarps][kAttnMaxGroup][kOPitch];  // after the chunks: per-warp partial O, then the merged heads
    };
    float part_o[kAttnMaxGroup][kHeadDim];        // this CTA's partial (unnormalised O), read by the cluster
    float part_m[kAttnMaxGroup];                  // its row max (-inf: no chunk)
    float part_l[kAttnMaxGroup];                  // its softmax sum
    float red_m[kAttnWarps][kAttnMaxGroup];
    float red_l[kAttnWarps][kAttnMaxGroup];
};

__device__ __forceinline__ void cp_async16_zfill(void* smem, const void* gmem, int src_bytes)
{
    const unsigned s = (unsigned) __cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(s), "l"(gmem), "r"(src_bytes) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* smem)
{
    const unsigned s = (unsigned) __cvta_generic_to_shared(smem);
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(s));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const void* smem)
{
    const unsigned s = (unsigned) __cvta_generic_to_shared(smem);
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(s));
}

__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1)
{
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
                 "{%8, %9}, {%0, %1, %2, %3};"
                 : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// (a, b) -> bf16x2 hi = rn(a, b) and lo = rn(a - hi_a, b - hi_b): hi + lo carries
// about 16 significant bits, so bf16 MMAs on both parts act like fp32 inputs
__device__ __forceinline__ void split_bf16(float a, float b, uint32_t& hi, uint32_t& lo)
{
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    const float2 hf = __bfloat1622float2(h);
    const __nv_bfloat162 l = __floats2bfloat162_rn(a - hf.x, b - hf.y);
    hi = *reinterpret_cast<const uint32_t*>(&h);
    lo = *reinterpret_cast<const uint32_t*>(&l);
}

// Cluster of csize CTAs per (row b, kv head); rank r takes the 64-position chunks
// r, r + csize, ... of positions 0..pos through a ring of kAttnBufs cp.async
// buffers whose first fill is requested before the dependency wait; one running
// max per warp and row, combined per CTA at the end.  Warp w owns positions 16w..16w+15 of a chunk.
// MMA fragments (lane = 4g + c): A rows g / g+8 = query heads of the group, B / C
// columns = positions (S) or head dims (O).  After the first cluster barrier rank
// r merges heads r, r + csize, ... from every rank's partial (distributed shared
// memory), normalises, rounds to fp16 and writes the o projection's rotated input
// (`ob` problem 0); the second barrier keeps every partial alive until then.
// Every CTA reaches both barriers (the only early exit is grid-uniform).
// With one row per sequence (qkv.nprob = 3) the kernel also does the RoPE/KV
// epilogue's work for its own (row, kv head) - the group's q head blocks and the k
// and v blocks, one warp each, read from the q/k/v matmul's partial sums - and a
// cluster barrier (release / acquire) makes q and the new K/V row visible to the
// cluster: one kernel fewer per layer.  (Several rows per sequence need every row's
// K/V before any row attends, across clusters; they keep the separate epilogue.)
__global__ __launch_bounds__(kAttnThreads) void exl3_dec_attn_kernel(const __grid_constant__ GvArgs ob,
                                                                     const __grid_constant__ DecAux x, int csize,
                                                                     const __grid_constant__ GvArgs qkv, int qkv_cb)
{
    griddep_launch();
    extern __shared__ __align__(128) unsigned char attn_smem_raw[];
    AttnSmem& sm = *reinterpret_cast<AttnSmem*>(attn_smem_raw);
    cg::cluster_group cluster = cg::this_cluster();
    const int rank = (int) cluster.block_rank();
    const int t = blockIdx.x / csize;
    const int kvh = t % x.kv_heads;
    const int b = t / x.kv_heads;  // row; its sequence b / rows_per_seq, position *pos + b % rows_per_seq
    // *pos and the cache rows before it were written before this step's kernels
    // (graph replays are separated by ordinary launches); only q and the new rows at
    // *pos .. *pos + rows_per_seq - 1 come from the RoPE epilogue this kernel depends on
    const long long pos0 = *x.pos;
    const long long pos = pos0 + b % x.rows_per_seq;
    const bool fused = qkv.nprob > 0;
    // a position past the cache: cluster-uniform; recorded in the device status by the
    // RoPE/KV epilogue's code (here, or in the separate kernel)
    const bool bad = pos0 < 0 || pos >= x.max_ctx;
    if (bad && !fused) return;
    const int L = bad ? 0 : (int) pos + 1;
    const int nch = (L + kDecChunk - 1) / kDecChunk;
    const int nloc = rank < nch ? (nch - 1 - rank) / csize + 1 : 0;
    const int group = x.q_heads / x.kv_heads;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, c = lane & 3;
    const GvProblem& po = gv_prob(ob, 0);
    if (tid < 2 * group && (tid >> 1) % csize == rank && po.suh)  // into L2: the o input scales of this rank's heads
        prefetch_l2_256(po.suh + (size_t) (kvh * group + (tid >> 1)) * 128, tid & 1);
    // fused: the q/k/v blocks of this warp - task tk < group is q head kvh * group + tk,
    // then k and v of head kvh; their output scales into L2 before the wait
    const int ntask = fused ? group + 2 : 0;
    for (int tk = rank * kAttnWarps + warp; tk < ntask; tk += kAttnWarps * csize) {
        const int pi = tk < group ? 0 : tk - group + 1;
        prefetch_l2_256(gv_prob(qkv, pi).svh + (size_t) (pi == 0 ? kvh * group + tk : kvh) * 128, lane);
    }

    const size_t hbase = (size_t) (b / x.rows_per_seq) * x.cache_b_stride + (size_t) kvh * x.cache_h_stride;
    // local chunk i -> buffer; rows >= its length are zero-filled; rows at positions
    // >= cut (this step's new rows) are left out for a load after the wait
    auto stage = [&](int i, int buf, long long cut) {
        const int p0 = (rank + i * csize) * kDecChunk;
        const int np = min(kDecChunk, L - p0);
        const __nv_bfloat16* kg = x.k_cache + hbase + (size_t) p0 * kHeadDim;
        const __nv_bfloat16* vg = x.v_cache + hbase + (size_t) p0 * kHeadDim;
        for (int e = tid; e < kDecChunk * 16; e += kAttnThreads) {
            const int row = e >> 4, seg = (e & 15) * 8;
            const bool ok = row < np;
            if (ok && p0 + row >= cut) continue;
            const size_t off = ok ? (size_t) row * kHeadDim + seg : 0;
            cp_async16_zfill(&sm.kv[buf][0][row][seg], kg + off, ok ? 16 : 0);
            cp_async16_zfill(&sm.kv[buf][1][row][seg], vg + off, ok ? 16 : 0);
        }
    };
    // first fill of the ring: rows written by earlier steps; the rows of positions
    // pos0 .. pos (this step's, from the RoPE epilogue) after the wait
    const int nfirst = min(nloc, kAttnBufs);
    for (int i = 0; i < nfirst; ++i) stage(i, i, pos0);
    griddep_wait();  // q (scaled) and the new K/V rows come from the RoPE epilogue, or the q/k/v matmul
    if (fused) {
        for (int tk = rank * kAttnWarps + warp; tk < ntask; tk += kAttnWarps * csize) {
            const int pi = tk < group ? 0 : tk - group + 1;
            const int nb = pi == 0 ? kvh * group + tk : kvh;
            const GvProblem& pp = gv_prob(qkv, pi);
            if (qkv_cb == 2) epi_block_row<2>(qkv, x, kEpiRopeKV, pi, pp, nullptr, nb, b, lane);
            else epi_block_row<0>(qkv, x, kEpiRopeKV, pi, pp, nullptr, nb, b, lane);
        }
        if (x.zero_ss && blockIdx.x == 0)  // the norm fold's duty of the skipped epilogue
            for (int i = tid; i < x.zero_rows; i += kAttnThreads) x.zero_ss[i] = 0.f;
        cluster.sync();  // release / acquire at cluster scope: the cluster's q and new K/V row are written
        if (bad) return;
    }
    for (int i = 0; i < nfirst; ++i) {
        const int p0 = (rank + i * csize) * kDecChunk;
        const int np = min(kDecChunk, L - p0);
        const int from = (int) max(0ll, pos0 - p0);
        for (int e = tid; e < (np - from) * 16; e += kAttnThreads) {
            const int row = from + (e >> 4), seg = (e & 15) * 8;
            const size_t off = hbase + (size_t) (p0 + row) * kHeadDim + seg;
            cp_async16_zfill(&sm.kv[i][0][row][seg], x.k_cache + off, 16);
            cp_async16_zfill(&sm.kv[i][1][row][seg], x.v_cache + off, 16);
        }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");

    // Q fragments of the group's heads (rows >= group are zero) as bf16 pairs
    // hi + lo (hi = bf16(q), lo = bf16(q - hi)): two MMAs give the scores to ~16 bits
    uint32_t qa[kHeadDim / 16][4], ql[kHeadDim / 16][4];
    {
        const float* qb = x.qbuf + ((size_t) b * x.q_heads + (size_t) kvh * group) * kHeadDim;
#pragma unroll
        for (int kk = 0; kk < kHeadDim / 16; ++kk)
#pragma unroll
            for (int hf = 0; hf < 2; ++hf) {
                const int row = g + 8 * hf;
                float2 f0 = make_float2(0.f, 0.f), f1 = make_float2(0.f, 0.f);
                if (row < group) {
                    f0 = *reinterpret_cast<const float2*>(qb + row * kHeadDim + 16 * kk + 2 * c);
                    f1 = *reinterpret_cast<const float2*>(qb + row * kHeadDim + 16 * kk + 2 * c + 8);
                }
                split_bf16(f0.x, f0.y, qa[kk][hf], ql[kk][hf]);
                split_bf16(f1.x, f1.y, qa[kk][2 + hf], ql[kk][2 + hf]);
            }
    }

    const int mi = lane >> 3, mr = lane & 7;  // ldmatrix: matrix and row this lane addresses
    float mg = -INFINITY, mh = -INFINITY;      // this warp's running row maxima (rows g, g+8)
    float lg = 0.f, lh = 0.f;                  // this thread's share of the warp's softmax sums
    float acc[kHeadDim / 8][4];
#pragma unroll
    for (int n = 0; n < kHeadDim / 8; ++n)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[n][e] = 0.f;

    for (int i = 0; i < nloc; ++i) {
        const int buf = i % kAttnBufs;
        // chunk i has landed: it is in the first fill (one group) or in the group of
        // iteration i - 2; after that only iteration i - 1's group may be pending
        if (i < 2) asm volatile("cp.async.wait_group 0;" ::: "memory");
        else asm volatile("cp.async.wait_group 1;" ::: "memory");
        __syncthreads();  // ... for every thread; and every warp is done with chunk i - 1
        if (i >= 1) {
            if (i + kAttnBufs - 1 < nloc) stage(i + kAttnBufs - 1, (i - 1) % kAttnBufs, LLONG_MAX);  // new rows included
            asm volatile("cp.async.commit_group;" ::: "memory");  // one group per iteration, maybe empty
        }
        const int np = min(kDecChunk, L - (rank + i * csize) * kDecChunk);

        // S = Q K^T over this warp's two 8-position tiles
        float s[2][4];
#pragma unroll
        for (int j = 0; j < 2; ++j)
#pragma unroll
            for (int e = 0; e < 4; ++e) s[j][e] = 0.f;
#pragma unroll
        for (int kk = 0; kk < kHeadDim / 16; ++kk) {
            uint32_t kb[4];
            ldsm_x4(kb, &sm.kv[buf][0][16 * warp + 8 * (mi >> 1) + mr][16 * kk + 8 * (mi & 1)]);
            mma_bf16_16816(s[0], qa[kk], kb[0], kb[1]);
            mma_bf16_16816(s[1], qa[kk], kb[2], kb[3]);
            mma_bf16_16816(s[0], ql[kk], kb[0], kb[1]);
            mma_bf16_16816(s[1], ql[kk], kb[2], kb[3]);
        }
        // mask positions past the context; the warp's new row maxima
        float ng = mg, nh = mh;
#pragma unroll
        for (int j = 0; j < 2; ++j)
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const bool ok = 16 * warp + 8 * j + 2 * c + e < np;
                s[j][e] = ok ? s[j][e] : -INFINITY;
                s[j][2 + e] = ok ? s[j][2 + e] : -INFINITY;
                ng = fmaxf(ng, s[j][e]);
                nh = fmaxf(nh, s[j][2 + e]);
            }
#pragma unroll
        for (int o = 1; o < 4; o <<= 1) {
            ng = fmaxf(ng, __shfl_xor_sync(0xffffffffu, ng, o));
            nh = fmaxf(nh, __shfl_xor_sync(0xffffffffu, nh, o));
        }
        if (ng == -INFINITY && nh == -INFINITY) continue;  // warp-uniform: no position of this warp is valid
        // rescale the running state to the new maxima (factor 0 on the first valid chunk)
        const float sg = __expf(mg - ng), sh = __expf(mh - nh);
        mg = ng;
        mh = nh;
        lg *= sg;
        lh *= sh;
#pragma unroll
        for (int n = 0; n < kHeadDim / 8; ++n) {
            acc[n][0] *= sg;
            acc[n][1] *= sg;
            acc[n][2] *= sh;
            acc[n][3] *= sh;
        }
        // P = exp(S - max) in fp32, fed to the MMA as bf16 pairs hi + lo
        uint32_t pa[4], pl[4];
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const float e0 = __expf(s[j][0] - mg), e1 = __expf(s[j][1] - mg);
            const float e2 = __expf(s[j][2] - mh), e3 = __expf(s[j][3] - mh);
            lg += e0 + e1;
            lh += e2 + e3;
            split_bf16(e0, e1, pa[2 * j], pl[2 * j]);
            split_bf16(e2, e3, pa[2 * j + 1], pl[2 * j + 1]);
        }
        // O += P V over the warp's 16 positions, 16 tiles of 8 head dims
#pragma unroll
        for (int q = 0; q < kHeadDim / 16; ++q) {
            uint32_t vb[4];
            ldsm_x4_t(vb, &sm.kv[buf][1][16 * warp + 8 * (mi & 1) + mr][16 * q + 8 * (mi >> 1)]);
            mma_bf16_16816(acc[2 * q], pa, vb[0], vb[1]);
            mma_bf16_16816(acc[2 * q + 1], pa, vb[2], vb[3]);
            mma_bf16_16816(acc[2 * q], pl, vb[0], vb[1]);
            mma_bf16_16816(acc[2 * q + 1], pl, vb[2], vb[3]);
        }
    }

    // this CTA's partial: the warps' states rescaled to the CTA's row maxima and summed
    __syncthreads();  // sm.o overlays the K/V ring, which other warps may still be reading
#pragma unroll
    for (int o = 1; o < 4; o <<= 1) {
        lg += __shfl_xor_sync(0xffffffffu, lg, o);
        lh += __shfl_xor_sync(0xffffffffu, lh, o);
    }
#pragma unroll
    for (int n = 0; n < kHeadDim / 8; ++n) {
        if (g < group) *reinterpret_cast<float2*>(&sm.o[warp][g][8 * n + 2 * c]) = make_float2(acc[n][0], acc[n][1]);
        if (g + 8 < group)
            *reinterpret_cast<float2*>(&sm.o[warp][g + 8][8 * n + 2 * c]) = make_float2(acc[n][2], acc[n][3]);
    }
    if (c == 0) {
        sm.red_m[warp][g] = mg;
        sm.red_m[warp][g + 8] = mh;
        sm.red_l[warp][g] = lg;
        sm.red_l[warp][g + 8] = lh;
    }
    __syncthreads();
    for (int hh = 0; hh < group; ++hh) {
        float m = sm.red_m[0][hh];
#pragma unroll
        for (int w = 1; w < kAttnWarps; ++w) m = fmaxf(m, sm.red_m[w][hh]);
        float v = 0.f, l = 0.f;
        if (m != -INFINITY) {
#pragma unroll
            for (int w = 0; w < kAttnWarps; ++w) {
                const float f = __expf(sm.red_m[w][hh] - m);
                v += f * sm.o[w][hh][tid];
                l += f * sm.red_l[w][hh];
            }
        }
        sm.part_o[hh][tid] = v;
        if (tid == 0) {
            sm.part_m[hh] = m;
            sm.part_l[hh] = l;
        }
    }
    cluster.sync();  // every rank's partial is complete

    // merge: rank r takes heads r, r + csize, ...; thread tid = head dim; ranks
    // without a chunk contribute max -inf, sum 0
    for (int hh = rank; hh < group; hh += csize) {
        float pm[kAttnMaxCluster], pv[kAttnMaxCluster], pl_[kAttnMaxCluster];
#pragma unroll
        for (int q = 0; q < kAttnMaxCluster; ++q) {
            if (q < csize) {
                const AttnSmem* rs = cluster.map_shared_rank(&sm, q);
                pm[q] = rs->part_m[hh];
                pl_[q] = rs->part_l[hh];
                pv[q] = rs->part_o[hh][tid];
            } else {
                pm[q] = -INFINITY;
                pl_[q] = 0.f;
                pv[q] = 0.f;
            }
        }
        float m = -INFINITY;
#pragma unroll
        for (int q = 0; q < kAttnMaxCluster; ++q) m = fmaxf(m, pm[q]);
        float l = 0.f, o = 0.f;
#pragma unroll
        for (int q = 0; q < kAttnMaxCluster; ++q) {
            const float f = __expf(pm[q] - m);
            l += f * pl_[q];
            o += f * pv[q];
        }
        sm.o[0][hh][tid] = __half2float(__float2half_rn(o / l));
    }
    // done reading the other ranks' partials: arrive now, wait before exiting
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
    __syncthreads();
    for (int j = warp;; j += kAttnWarps) {
        const int hh = rank + j * csize;
        if (hh >= group) break;
        float xv[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) xv[i] = sm.o[0][hh][lane + 32 * i];
        store_rotated(po.xd, po.sblk, po.suh, po.k, b, kvh * group + hh, lane, xv);
    }
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");  // partials stay readable until every rank has merged
}

// h += y and the row's sum of squares (tensor-parallel path, after the all-reduce)
__global__ __launch_bounds__(256) void exl3_dec_residual_kernel(float* __restrict__ h, long long h_stride,
                                                                const float* __restrict__ y, long long y_stride,
                                                                float* __restrict__ ss, int batch, int hidden)
{
    griddep_launch();
    griddep_wait();
    const int lane = threadIdx.x & 31;
    const int nblk = hidden >> 7;
    const int warps = gridDim.x * (blockDim.x >> 5);
    for (int task = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); task < batch * nblk; task += warps) {
        const int r = task / nblk, b = task - r * nblk;
        float* hr = h + (size_t) r * h_stride + b * 128;
        const float* yr = y + (size_t) r * y_stride + b * 128;
        float sq = 0.f;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const float nv = hr[lane + 32 * e] + yr[lane + 32 * e];
            hr[lane + 32 * e] = nv;
            sq += nv * nv;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
        if (lane == 0) atomicAdd(ss + r, sq);
    }
}

// Tensor-parallel output epilogue with the exchange folded in (o / down projection,
// one launch per sub-layer).  Each warp, per (row, block) task: finishes the block
// row, stores each fp32 partial with the call's tag (bit 31, the buffer's
// generation, the call epoch) in one 8-byte store into this rank's slot of every
// rank's peer buffer (NVLink), then reads every rank's slots of the same block row
// from its own buffer until each carries the tag - a reader that sees the tag sees
// the value, so no fence and no arrival counter - bounded by 2 s of %globaltimer;
// then h += the sum, the row's sum of squares, and (norm fold) the next sub-layer's
// inputs.  A warp whose wait gives up records EXL3B200_ETIMEOUT and poisons the
// buffer: later block rows are not updated, the epoch is not advanced, and every
// later launch on the buffer returns at once with EXL3B200_ETIMEOUT until the host
// re-arms it (exl3b200_peer_reset, which also advances the generation so that
// slots written before it never match).  The last CTA to finish advances the
// epoch.  The grid is at most one CTA per SM, so every CTA is resident while it
// waits, and it is the same on every rank (same shapes).  Slots alternate between
// two parities by call; a rank cannot reach call k+2 before every peer has finished
// call k (its call k+1 values only leave after its call k epilogue ended).
template <int CB>
__global__ __launch_bounds__(256) void exl3_dec_peer_epilogue_kernel(const __grid_constant__ GvArgs a,
                                                                     const __grid_constant__ DecAux x)
{
    griddep_launch();
    const int lane = threadIdx.x & 31;
    gv_prefetch_epilogue(a, lane);
    if (x.fold_n) {
        const int task = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
        if (task < a.out_tasks) fold_prefetch(x, task % (gv_prob(a, 0).n >> 7), lane);
    }
    griddep_wait();
    PeerCtl* ctl = reinterpret_cast<PeerCtl*>(x.peer[x.peer_rank]);
    // an earlier exchange gave up: the partial sums are still consumed (the matmul
    // state is left zeroed for the next call), but nothing is stored or updated
    const bool poisoned = *reinterpret_cast<volatile unsigned int*>(&ctl->poisoned) != 0u;
    const unsigned int epoch = *reinterpret_cast<volatile unsigned int*>(&ctl->epoch) + 1u;
    const unsigned int parity = epoch & 1u;
    const unsigned int gen = *reinterpret_cast<volatile unsigned int*>(x.peer[x.peer_rank] + kPeerGen);
    // call tag: bit 31 set (zeroed slots never match), generation, call epoch
    const unsigned int tag = 0x80000000u | ((gen & 0x7fu) << 24) | (epoch & 0xffffffu);
    const int warps = gridDim.x * (blockDim.x >> 5);
    const int task0 = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    bool gave_up = false;
    for (int task = task0; task < a.out_tasks; task += warps) {
        const GvProblem& p = gv_prob(a, 0);
        const int nblocks = p.n >> 7;
        const int r = task / nblocks, nb = task - r * nblocks;
        FoldPre fp;
        if (x.fold_n) fold_preload(x, r, nb, lane, fp);
        float v[4];
        gv_finish<CB>(p, nb, r, lane, v);
        if (poisoned || gave_up) continue;
        // this rank's block row into its slot of every rank's buffer, then every rank's
        // slot of the same block row from this rank's own buffer, each as soon as its tag
        // shows (per warp: no grid-wide wait)
        for (int q = 0; q < x.peer_world; ++q) {
            unsigned long long* dst = peer_slot(x, q, parity, x.peer_rank, r) + nb * 128;
#pragma unroll
            for (int e = 0; e < 4; ++e) st_slot_sys(dst + lane + 32 * e, v[e], tag);
        }
        float sum[4] = {0.f, 0.f, 0.f, 0.f};
        bool ok = true;
        const unsigned long long t0 = globaltimer_ns();
        for (int q = 0; q < x.peer_world && ok; ++q) {
            const unsigned long long* src = peer_slot(x, x.peer_rank, parity, q, r) + nb * 128;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                unsigned long long w = ld_slot_sys(src + lane + 32 * e);
                while ((unsigned int) (w >> 32) != tag) {
                    if (globaltimer_ns() - t0 > x.peer_wait_ns) {
                        ok = false;
                        break;
                    }
                    w = ld_slot_sys(src + lane + 32 * e);
                }
                if (!ok) break;
                sum[e] += __uint_as_float((unsigned int) w);
            }
        }
        if (!__all_sync(0xffffffffu, ok)) {
            // a rank did not answer in time: status, poison; this and later block rows
            // of this warp are not updated (h is left partly updated: the step is lost)
            if (lane == 0) {
                if (x.status) atomicCAS(x.status, 0, (int) kErrTimeout);
                atomicExch(&ctl->poisoned, 1u);
            }
            gave_up = true;
            continue;
        }
        float* hr = x.resid + (size_t) r * x.resid_stride + nb * 128;
        float sq = 0.f;
        float nv[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            nv[e] = hr[lane + 32 * e] + sum[e];
            hr[lane + 32 * e] = nv[e];
            sq += nv[e] * nv[e];
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
        if (lane == 0) atomicAdd(x.ss_acc + r, sq);
        if (x.fold_n) fold_out(x, r, nb, lane, nv, fp);
    }
    if (poisoned && threadIdx.x == 0 && x.status) atomicCAS(x.status, 0, (int) kErrTimeout);
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        if (atomicAdd(&ctl->done, 1u) == gridDim.x - 1) {
            ctl->done = 0u;
            if (!*reinterpret_cast<volatile unsigned int*>(&ctl->poisoned)) {
                __threadfence();
                *reinterpret_cast<volatile unsigned int*>(&ctl->epoch) = epoch;
            }
        }
    }
}

__global__ void exl3_peer_reset_kernel(char* buf)
{
    unsigned int* w = reinterpret_cast<unsigned int*>(buf);
    const unsigned int gen = w[kPeerGen / 4];
    for (int i = 0; i < (int) (kPeerData / 4); ++i) w[i] = 0u;
    w[kPeerGen / 4] = gen + 1u;
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
template <typename Kern, typename... Args>
static int dec_launch(Kern kern, int grid, int block, cudaStream_t stream, Args... args)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned) std::max(grid, 1));
    cfg.blockDim = dim3((unsigned) block);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, args...) == cudaSuccess ? kOk : kErrLaunch;
}

// The attention kernel: shared memory beyond the 48 KB default and clusters of up
// to 16 CTAs (beyond the portable 8), set once per device; the cluster size is the
// largest power of two <= min(16, chunks of the cache) that the device can hold.
static int dec_attn_setup(int max_chunks, int* csize, int* max_clusters = nullptr)
{
    static int done[64] = {0};
    static int fits[64][5] = {{0}};    // per device, cluster size 1, 2, 4, 8, 16: 0 unknown, 1 yes, 2 no
    static int resident[64][5] = {{0}};  // clusters of that size the device holds at once
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return kErrLaunch;
    if (!done[dev]) {
        if (cudaFuncSetAttribute(exl3_dec_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int) sizeof(AttnSmem)) != cudaSuccess ||
            cudaFuncSetAttribute(exl3_dec_attn_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) !=
                cudaSuccess)
            return kErrLaunch;
        done[dev] = 1;
    }
    int c = 1, li = 0;
    while (c * 2 <= std::min(kAttnMaxCluster, max_chunks)) {
        c *= 2;
        ++li;
    }
    for (; c >= 1; c /= 2, --li) {
        if (!fits[dev][li]) {
            cudaLaunchConfig_t cfg = {};
            cfg.gridDim = dim3((unsigned) c);
            cfg.blockDim = dim3((unsigned) kAttnThreads);
            cfg.dynamicSmemBytes = sizeof(AttnSmem);
            cudaLaunchAttribute attr[1];
            attr[0].id = cudaLaunchAttributeClusterDimension;
            attr[0].val.clusterDim.x = (unsigned) c;
            attr[0].val.clusterDim.y = 1;
            attr[0].val.clusterDim.z = 1;
            cfg.attrs = attr;
            cfg.numAttrs = 1;
            int n = 0;
            fits[dev][li] = (cudaOccupancyMaxActiveClusters(&n, exl3_dec_attn_kernel, &cfg) == cudaSuccess && n > 0)
                                ? 1 : 2;
            resident[dev][li] = n;
        }
        if (fits[dev][li] == 1) {
            *csize = c;
            if (max_clusters) *max_clusters = resident[dev][li];
            return kOk;
        }
    }
    return kErrLaunch;
}

static int dec_launch_attn(const GvArgs& ob, const DecAux& x, int groups, cudaStream_t stream,
                           const GvArgs* qkv = nullptr, int qkv_cb = 0)
{
    int csize = 1;
    const int rc = dec_attn_setup((x.max_ctx + kDecChunk - 1) / kDecChunk, &csize);
    if (rc != kOk) return rc;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned) (groups * csize));
    cfg.blockDim = dim3((unsigned) kAttnThreads);
    cfg.dynamicSmemBytes = sizeof(AttnSmem);
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = (unsigned) csize;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    GvArgs none = {};  // nprob 0: q, k and v were finished by the RoPE/KV epilogue
    return cudaLaunchKernelEx(&cfg, exl3_dec_attn_kernel, ob, x, csize, qkv ? *qkv : none, qkv_cb) == cudaSuccess
               ? kOk
               : kErrLaunch;
}

static int dec_grid(int tasks) { return std::min((tasks + 7) / 8, 8 * gv_sm_count()); }

template <int MODE>
static int dec_launch_epilogue(const GvArgs& a, const DecAux& x, int cb, cudaStream_t st)
{
    const int g = dec_grid(a.out_tasks);
    return cb == 2 ? dec_launch(exl3_dec_epilogue_kernel<2, MODE>, g, 256, st, a, x)
                   : dec_launch(exl3_dec_epilogue_kernel<0, MODE>, g, 256, st, a, x);
}

static size_t al256(size_t v) { return (v + 255) & ~(size_t) 255; }

static bool dec_linear_ok(const exl3b200_linear* l, int k, int n)
{
    return l && l->trellis && l->suh && l->svh && l->k == k && l->n == n && !((uintptr_t) l->trellis & 3);
}

static void dec_problem(GvProblem& p, const exl3b200_linear* l, int m, uint32_t* xd, float* sblk, float* acc)
{
    p = GvProblem{};
    p.trellis = reinterpret_cast<const uint32_t*>(l->trellis);
    p.suh = reinterpret_cast<const __half*>(l->suh);
    p.svh = reinterpret_cast<const __half*>(l->svh);
    p.xd = xd;
    p.sblk = sblk;
    p.acc = acc;
    p.acc_nb_stride = 16 * 128;
    p.k = l->k;
    p.n = l->n;
    p.m = m;
}

// Workspace layout of the attention sub-layer.
struct DecAttnLayout {
    size_t st_q, st_k, st_v, st_o, state_bytes;
    size_t xd_q, xd_k, xd_v, sb_q, sb_k, sb_v, qbuf, xd_o, sb_o, scratch_bytes;
};

static DecAttnLayout dec_attn_layout(int batch, int hidden, int q_heads, int kv_heads, int max_ctx)
{
    DecAttnLayout L = {};
    const int nq = q_heads * kHeadDim, nkv = kv_heads * kHeadDim;
    size_t o = 0;
    L.st_q = o; o += gv_state_bytes_per_problem(nq);
    L.st_k = o; o += gv_state_bytes_per_problem(nkv);
    L.st_v = o; o += gv_state_bytes_per_problem(nkv);
    L.st_o = o; o += gv_state_bytes_per_problem(hidden);
    L.state_bytes = o;
    o = 0;
    L.xd_q = o; o += gv_xd_bytes(batch, hidden);
    L.xd_k = o; o += gv_xd_bytes(batch, hidden);
    L.xd_v = o; o += gv_xd_bytes(batch, hidden);
    L.sb_q = o; o += gv_sblk_bytes(batch, hidden);
    L.sb_k = o; o += gv_sblk_bytes(batch, hidden);
    L.sb_v = o; o += gv_sblk_bytes(batch, hidden);
    L.qbuf = o; o += al256((size_t) batch * nq * sizeof(float));
    L.xd_o = o; o += gv_xd_bytes(batch, nq);
    L.sb_o = o; o += gv_sblk_bytes(batch, nq);
    L.scratch_bytes = o;
    return L;
}

struct DecMlpLayout {
    size_t st_g, st_u, st_d, state_bytes;
    size_t xd_g, xd_u, sb_g, sb_u, xd_d, sb_d, scratch_bytes;
};

static DecMlpLayout dec_mlp_layout(int batch, int hidden, int inter)
{
    DecMlpLayout L = {};
    size_t o = 0;
    L.st_g = o; o += gv_state_bytes_per_problem(inter);
    L.st_u = o; o += gv_state_bytes_per_problem(inter);
    L.st_d = o; o += gv_state_bytes_per_problem(hidden);
    L.state_bytes = o;
    o = 0;
    L.xd_g = o; o += gv_xd_bytes(batch, hidden);
    L.xd_u = o; o += gv_xd_bytes(batch, hidden);
    L.sb_g = o; o += gv_sblk_bytes(batch, hidden);
    L.sb_u = o; o += gv_sblk_bytes(batch, hidden);
    L.xd_d = o; o += gv_xd_bytes(batch, inter);
    L.sb_d = o; o += gv_sblk_bytes(batch, inter);
    L.scratch_bytes = o;
    return L;
}

// Norm fold into a sub-layer's residual epilogue: the next sub-layer's inputs.
struct DecFoldOut {
    int n;
    FoldTarget t[kFoldMax];
    const void* norm_w;  // bf16 [hidden]
    float* fold_c;       // [rows]
};

// Workspace of a whole layer with the norm fold: the attention sub-layer's, the
// MLP sub-layer's, and the per-row pre-scale the residual epilogues write.
struct DecLayerLayout {
    DecAttnLayout A;
    DecMlpLayout M;
    size_t fold_c, state_bytes, scratch_bytes;
};

static DecLayerLayout dec_layer_layout(int rows, int hidden, int q_heads, int kv_heads, int inter, int max_ctx)
{
    DecLayerLayout L = {};
    L.A = dec_attn_layout(rows, hidden, q_heads, kv_heads, max_ctx);
    L.M = dec_mlp_layout(rows, hidden, inter);
    L.state_bytes = L.A.state_bytes + L.M.state_bytes;
    L.fold_c = L.A.scratch_bytes + L.M.scratch_bytes;
    L.scratch_bytes = L.fold_c + al256((size_t) rows * sizeof(float));
    return L;
}

// Final epilogue of a sub-layer: residual add into h (+ sum of squares), or an
// fp32 store of the partial for a tensor-parallel all-reduce.  x arrives with the
// consumer-side fold fields cleared; fold (optional) is applied to the residual.
static int dec_finish(GvArgs& a, DecAux& x, int cb, float* h, long long h_stride, float* ss_out, float* y_out,
                      long long y_stride, const exl3b200_peers* peers, int batch, int hidden, cudaStream_t st,
                      const DecFoldOut* fold = nullptr)
{
    x.fold_c_in = nullptr;
    x.zero_ss = nullptr;
    if (fold && fold->n > 0) {
        if (y_out) return kErrBadArgument;  // the all-reduce path finishes the residual outside
        x.fold_n = fold->n;
        for (int i = 0; i < kFoldMax; ++i) x.fold[i] = i < fold->n ? fold->t[i] : FoldTarget{};
        x.fold_norm_w = reinterpret_cast<const __nv_bfloat16*>(fold->norm_w);
        x.fold_c = fold->fold_c;
    }
    if (peers) {
        for (int q = 0; q < kPeerMaxRanks; ++q) x.peer[q] = q < peers->world ? (char*) peers->buffers[q] : nullptr;
        x.peer_world = peers->world;
        x.peer_rank = peers->rank;
        x.peer_rows = peers->max_rows;
        x.peer_hidden = peers->hidden;
        x.peer_wait_ns = wait_limit_ns(kPeerTimeoutNs);
        x.status = exl3_status_dev_ptr();
        x.resid = h;
        x.resid_stride = h_stride;
        x.ss_acc = ss_out;
        const int g = std::min(dec_grid(a.out_tasks), gv_sm_count());  // resident: its CTAs wait on each other
        return cb == 2 ? dec_launch(exl3_dec_peer_epilogue_kernel<2>, g, 256, st, a, x)
                       : dec_launch(exl3_dec_peer_epilogue_kernel<0>, g, 256, st, a, x);
    }
    if (y_out) {
        a.inl[0].out = y_out;
        a.inl[0].out_stride = y_stride;
        a.out_dtype = 2;
        a.epi_mode = kEpiStore;
        return gv_launch_epilogue(a, cb, a.out_tasks, true, st);
    }
    x.resid = h;
    x.resid_stride = h_stride;
    x.ss_acc = ss_out;
    return dec_launch_epilogue<kEpiResidual>(a, x, cb, st);
}

static int dec_common_checks(int batch, int hidden, int K, int cb, const float* h, long long h_stride,
                             const float* ss_in, const float* ss_out, const void* norm_w, const void* state,
                             const void* scratch)
{
    if (!h || !ss_in || !ss_out || !norm_w || !state || !scratch) return kErrNullPointer;
    if (batch < 1 || batch > EXL3B200_GEMV_MAX_M || hidden <= 0 || hidden % 128 || h_stride < hidden)
        return kErrBadShape;
    if (K < 2 || K > 4) return kErrBadBits;
    if (cb < 0 || cb > 2) return kErrBadCodebook;
    if (((uintptr_t) state & 255) || ((uintptr_t) scratch & 255)) return kErrUnaligned;
    return kOk;
}

static int dec_peers_check(const exl3b200_peers* peers, int batch, int hidden)
{
    if (!peers) return kOk;
    if (peers->world < 1 || peers->world > kPeerMaxRanks || peers->rank < 0 || peers->rank >= peers->world)
        return kErrBadArgument;
    if (peers->max_rows < batch || peers->hidden != hidden) return kErrBadShape;
    for (int q = 0; q < peers->world; ++q) {
        if (!peers->buffers[q]) return kErrNullPointer;
        if ((uintptr_t) peers->buffers[q] & 255) return kErrUnaligned;
    }
    return kOk;
}

}  // namespace exl3b200

using namespace exl3b200;

extern "C" size_t exl3b200_peer_buffer_size(int max_rows, int hidden)
{
    if (max_rows < 1 || hidden <= 0 || hidden % 128) return 0;
    return kPeerData + (size_t) 2 * kPeerMaxRanks * max_rows * hidden * sizeof(unsigned long long);
}

extern "C" int exl3b200_peer_buffer_alloc(size_t bytes, void** ptr, void* ipc_handle)
{
    if (!ptr || !ipc_handle) return kErrNullPointer;
    if (bytes < kPeerData) return kErrBadShape;
    void* p = nullptr;
    if (cudaMalloc(&p, bytes) != cudaSuccess) return kErrLaunch;
    cudaIpcMemHandle_t h;
    if (cudaMemset(p, 0, bytes) != cudaSuccess || cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
        cudaFree(p);
        return kErrLaunch;
    }
    memcpy(ipc_handle, &h, sizeof(h));
    *ptr = p;
    return kOk;
}

extern "C" int exl3b200_peer_buffer_open(const void* ipc_handle, void** ptr)
{
    if (!ptr || !ipc_handle) return kErrNullPointer;
    cudaIpcMemHandle_t h;
    memcpy(&h, ipc_handle, sizeof(h));
    return cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess ? kOk : kErrLaunch;
}

extern "C" int exl3b200_peer_buffer_close(void* ptr)
{
    if (!ptr) return kErrNullPointer;
    return cudaIpcCloseMemHandle(ptr) == cudaSuccess ? kOk : kErrLaunch;
}

extern "C" int exl3b200_peer_reset(void* own_buffer, void* stream)
{
    if (!own_buffer) return kErrNullPointer;
    if ((uintptr_t) own_buffer & 255) return kErrUnaligned;
    // control block zeroed (the exchange's and the expert-parallel exchange's counters,
    // epochs and poison word), the generation advanced: slots written before the reset
    // carry older tags and are never taken for this generation's calls
    exl3_peer_reset_kernel<<<1, 1, 0, reinterpret_cast<cudaStream_t>(stream)>>>(reinterpret_cast<char*>(own_buffer));
    return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;
}

extern "C" int exl3b200_peer_buffer_free(void* ptr)
{
    if (!ptr) return kErrNullPointer;
    return cudaFree(ptr) == cudaSuccess ? kOk : kErrLaunch;
}

extern "C" int exl3b200_decode_attention_workspace(int batch, int hidden, int q_heads, int kv_heads, int max_ctx,
                                                   size_t* state_bytes, size_t* scratch_bytes)
{
    if (!state_bytes || !scratch_bytes) return kErrNullPointer;
    if (batch < 1 || batch > EXL3B200_GEMV_MAX_M || hidden <= 0 || hidden % 128 || q_heads < 1 || kv_heads < 1 ||
        q_heads % kv_heads || q_heads / kv_heads > kAttnMaxGroup || max_ctx < 1)
        return kErrBadShape;
    const DecAttnLayout L = dec_attn_layout(batch, hidden, q_heads, kv_heads, max_ctx);
    *state_bytes = L.state_bytes;
    *scratch_bytes = L.scratch_bytes;
    return kOk;
}

extern "C" int exl3b200_decode_mlp_workspace(int batch, int hidden, int inter, size_t* state_bytes,
                                             size_t* scratch_bytes)
{
    if (!state_bytes || !scratch_bytes) return kErrNullPointer;
    if (batch < 1 || batch > EXL3B200_GEMV_MAX_M || hidden <= 0 || hidden % 128 || inter <= 0 || inter % 128)
        return kErrBadShape;
    const DecMlpLayout L = dec_mlp_layout(batch, hidden, inter);
    *state_bytes = L.state_bytes;
    *scratch_bytes = L.scratch_bytes;
    return kOk;
}

// batch rows; rows r = R s + j of sequence s (cache slot s) at position *pos + j.
static int dec_attention(int batch, int rows_per_seq, int hidden, int q_heads, int kv_heads, int K, int cb, float* h,
                         long long h_stride, const float* ss_in, float* ss_out, const void* norm_w, float eps,
                         const exl3b200_linear* q, const exl3b200_linear* k, const exl3b200_linear* v,
                         const exl3b200_linear* o, void* k_cache, void* v_cache, int max_ctx, const long long* pos,
                         const float* inv_freq, float* y_out, long long y_stride, const exl3b200_peers* peers,
                         void* state, size_t state_bytes, void* scratch, size_t scratch_bytes, void* stream,
                         const float* fold_c_in = nullptr, const DecFoldOut* fold_out = nullptr)
{
    if (rows_per_seq < 1 || batch % rows_per_seq) return kErrBadShape;
    int rc = dec_common_checks(batch, hidden, K, cb, h, h_stride, ss_in, ss_out, norm_w, state, scratch);
    if (rc != kOk) return rc;
    rc = dec_peers_check(peers, batch, hidden);
    if (rc != kOk) return rc;
    if (!k_cache || !v_cache || !pos || !inv_freq) return kErrNullPointer;
    if (q_heads < 1 || kv_heads < 1 || q_heads % kv_heads || q_heads / kv_heads > kAttnMaxGroup || max_ctx < 1)
        return kErrBadShape;
    const int nq = q_heads * kHeadDim, nkv = kv_heads * kHeadDim;
    if (!dec_linear_ok(q, hidden, nq) || !dec_linear_ok(k, hidden, nkv) || !dec_linear_ok(v, hidden, nkv) ||
        !dec_linear_ok(o, nq, hidden))
        return kErrBadShape;
    if (y_out && y_stride < hidden) return kErrBadShape;
    if (((uintptr_t) k_cache & 15) || ((uintptr_t) v_cache & 15)) return kErrUnaligned;
    const DecAttnLayout L = dec_attn_layout(batch, hidden, q_heads, kv_heads, max_ctx);
    if (state_bytes < L.state_bytes || scratch_bytes < L.scratch_bytes) return kErrWorkspace;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    char* S = reinterpret_cast<char*>(state);
    char* W = reinterpret_cast<char*>(scratch);
    const bool mul1 = cb == 2;

    DecAux x = {};
    x.h = h;
    x.h_stride = h_stride;
    x.ss_in = ss_in;
    x.ss_out = ss_out;
    x.zero_rows = batch;
    x.norm_w = reinterpret_cast<const __nv_bfloat16*>(norm_w);
    x.eps = eps;
    x.inv_hidden = 1.f / (float) hidden;
    x.pos = pos;
    x.inv_freq = inv_freq;
    x.status = exl3_status_dev_ptr();
    x.qbuf = reinterpret_cast<float*>(W + L.qbuf);
    x.k_cache = reinterpret_cast<__nv_bfloat16*>(k_cache);
    x.v_cache = reinterpret_cast<__nv_bfloat16*>(v_cache);
    x.cache_h_stride = (long long) max_ctx * kHeadDim;
    x.cache_b_stride = (long long) kv_heads * x.cache_h_stride;
    x.max_ctx = max_ctx;
    x.q_heads = q_heads;
    x.kv_heads = kv_heads;
    x.rows_per_seq = rows_per_seq;

    // 1-3: norm input stage, q/k/v matmul, RoPE + KV append epilogue
    GvArgs a = {};
    a.nprob = 3;
    dec_problem(a.inl[0], q, batch, reinterpret_cast<uint32_t*>(W + L.xd_q),
                mul1 ? reinterpret_cast<float*>(W + L.sb_q) : nullptr, reinterpret_cast<float*>(S + L.st_q));
    dec_problem(a.inl[1], k, batch, reinterpret_cast<uint32_t*>(W + L.xd_k),
                mul1 ? reinterpret_cast<float*>(W + L.sb_k) : nullptr, reinterpret_cast<float*>(S + L.st_k));
    dec_problem(a.inl[2], v, batch, reinterpret_cast<uint32_t*>(W + L.xd_v),
                mul1 ? reinterpret_cast<float*>(W + L.sb_v) : nullptr, reinterpret_cast<float*>(S + L.st_v));
    gv_prefix_inline(a);
    DecAux xe = x;  // the RoPE epilogue's view: with the norm fold it scales and zeroes ss_out
    if (fold_c_in) {
        // the previous sub-layer's residual epilogue wrote the q/k/v inputs
        xe.fold_c_in = fold_c_in;
        xe.zero_ss = ss_out;
    } else {
        rc = dec_launch(exl3_dec_input_kernel, dec_grid(a.in_tasks), 256, st, a, x);
        if (rc != kOk) return rc;
    }
    rc = gv_launch_matmul(a, K, cb, batch, 0, true, st);
    if (rc != kOk) return rc;
    // one row per sequence and every cluster resident at once: the attention kernel
    // finishes q/k/v itself (with more clusters than one wave, each later wave would
    // pay the finishing round trips again; the separate epilogue spreads them over
    // the whole GPU once)
    int csize = 1, max_clusters = 0;
    rc = dec_attn_setup((max_ctx + kDecChunk - 1) / kDecChunk, &csize, &max_clusters);
    if (rc != kOk) return rc;
    const bool rope_in_attn = rows_per_seq == 1 && batch * kv_heads <= max_clusters;
    if (!rope_in_attn) {
        rc = dec_launch_epilogue<kEpiRopeKV>(a, xe, cb, st);
        if (rc != kOk) return rc;
    }

    // 4: attention (a cluster per row and kv head; its merge writes the o input)
    GvArgs b = {};
    b.nprob = 1;
    dec_problem(b.inl[0], o, batch, reinterpret_cast<uint32_t*>(W + L.xd_o),
                mul1 ? reinterpret_cast<float*>(W + L.sb_o) : nullptr, reinterpret_cast<float*>(S + L.st_o));
    gv_prefix_inline(b);
    rc = rope_in_attn ? dec_launch_attn(b, xe, batch * kv_heads, st, &a, cb == 2 ? 2 : 0)
                      : dec_launch_attn(b, x, batch * kv_heads, st);
    if (rc != kOk) return rc;

    // 5-6: o matmul, residual (or fp32 partial for the all-reduce)
    rc = gv_launch_matmul(b, K, cb, batch, 0, true, st);
    if (rc != kOk) return rc;
    return dec_finish(b, x, cb, h, h_stride, ss_out, y_out, y_stride, peers, batch, hidden, st, fold_out);
}

extern "C" int exl3b200_decode_attention(int batch, int hidden, int q_heads, int kv_heads, int K, int cb, float* h,
                                         long long h_stride, const float* ss_in, float* ss_out, const void* norm_w,
                                         float eps, const exl3b200_linear* q, const exl3b200_linear* k,
                                         const exl3b200_linear* v, const exl3b200_linear* o, void* k_cache,
                                         void* v_cache, int max_ctx, const long long* pos, const float* inv_freq,
                                         float* y_out, long long y_stride, const exl3b200_peers* peers, void* state,
                                         size_t state_bytes, void* scratch, size_t scratch_bytes, void* stream)
{
    return dec_attention(batch, 1, hidden, q_heads, kv_heads, K, cb, h, h_stride, ss_in, ss_out, norm_w, eps, q, k,
                         v, o, k_cache, v_cache, max_ctx, pos, inv_freq, y_out, y_stride, peers, state, state_bytes,
                         scratch, scratch_bytes, stream);
}

extern "C" int exl3b200_decode_attention_rows(int rows, int rows_per_seq, int hidden, int q_heads, int kv_heads,
                                              int K, int cb, float* h, long long h_stride, const float* ss_in,
                                              float* ss_out, const void* norm_w, float eps, const exl3b200_linear* q,
                                              const exl3b200_linear* k, const exl3b200_linear* v,
                                              const exl3b200_linear* o, void* k_cache, void* v_cache, int max_ctx,
                                              const long long* pos, const float* inv_freq, float* y_out,
                                              long long y_stride, const exl3b200_peers* peers, void* state,
                                              size_t state_bytes, void* scratch, size_t scratch_bytes, void* stream)
{
    return dec_attention(rows, rows_per_seq, hidden, q_heads, kv_heads, K, cb, h, h_stride, ss_in, ss_out, norm_w,
                         eps, q, k, v, o, k_cache, v_cache, max_ctx, pos, inv_freq, y_out, y_stride, peers, state,
                         state_bytes, scratch, scratch_bytes, stream);
}

static int dec_mlp(int batch, int hidden, int inter, int K, int cb, float* h, long long h_stride, const float* ss_in,
                   float* ss_out, const void* norm_w, float eps, const exl3b200_linear* gate,
                   const exl3b200_linear* up, const exl3b200_linear* down, float swiglu_limit, float* y_out,
                   long long y_stride, const exl3b200_peers* peers, void* state, size_t state_bytes, void* scratch,
                   size_t scratch_bytes, void* stream, const float* fold_c_in = nullptr,
                   const DecFoldOut* fold_out = nullptr)
{
    int rc = dec_common_checks(batch, hidden, K, cb, h, h_stride, ss_in, ss_out, norm_w, state, scratch);
    if (rc != kOk) return rc;
    rc = dec_peers_check(peers, batch, hidden);
    if (rc != kOk) return rc;
    if (inter <= 0 || inter % 128) return kErrBadShape;
    if (!dec_linear_ok(gate, hidden, inter) || !dec_linear_ok(up, hidden, inter) || !dec_linear_ok(down, inter, hidden))
        return kErrBadShape;
    if (y_out && y_stride < hidden) return kErrBadShape;
    const DecMlpLayout L = dec_mlp_layout(batch, hidden, inter);
    if (state_bytes < L.state_bytes || scratch_bytes < L.scratch_bytes) return kErrWorkspace;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    char* S = reinterpret_cast<char*>(state);
    char* W = reinterpret_cast<char*>(scratch);
    const bool mul1 = cb == 2;

    DecAux x = {};
    x.h = h;
    x.h_stride = h_stride;
    x.ss_in = ss_in;
    x.ss_out = ss_out;
    x.zero_rows = batch;
    x.norm_w = reinterpret_cast<const __nv_bfloat16*>(norm_w);
    x.eps = eps;
    x.inv_hidden = 1.f / (float) hidden;

    GvArgs a = {};
    a.nprob = 2;
    dec_problem(a.inl[0], gate, batch, reinterpret_cast<uint32_t*>(W + L.xd_g),
                mul1 ? reinterpret_cast<float*>(W + L.sb_g) : nullptr, reinterpret_cast<float*>(S + L.st_g));
    dec_problem(a.inl[1], up, batch, reinterpret_cast<uint32_t*>(W + L.xd_u),
                mul1 ? reinterpret_cast<float*>(W + L.sb_u) : nullptr, reinterpret_cast<float*>(S + L.st_u));
    // the SwiGLU epilogue of gate writes the rotated input of down
    a.inl[0].out = W + L.xd_d;
    a.inl[0].out_stride = inter;
    a.inl[0].out_suh = reinterpret_cast<const __half*>(down->suh);
    a.inl[0].out_sblk = mul1 ? reinterpret_cast<float*>(W + L.sb_d) : nullptr;
    gv_prefix_inline(a);
    DecAux xe = x;  // the SwiGLU epilogue's view: with the norm fold it scales and zeroes ss_out
    if (fold_c_in) {
        xe.fold_c_in = fold_c_in;
        xe.zero_ss = ss_out;
    } else {
        rc = dec_launch(exl3_dec_input_kernel, dec_grid(a.in_tasks), 256, st, a, x);
        if (rc != kOk) return rc;
    }
    rc = gv_launch_matmul(a, K, cb, batch, 0, true, st);
    if (rc != kOk) return rc;

    GvArgs e = a;
    e.stride = 2;
    e.offset = 0;
    e.nprob = 1;
    e.out_tasks = batch * (inter / 128);
    e.epi_mode = kEpiSwiglu;
    e.swiglu_limit = swiglu_limit;
    rc = dec_launch_epilogue<kEpiSwiglu>(e, xe, cb, st);
    if (rc != kOk) return rc;

    GvArgs d = {};
    d.nprob = 1;
    dec_problem(d.inl[0], down, batch, reinterpret_cast<uint32_t*>(W + L.xd_d),
                mul1 ? reinterpret_cast<float*>(W + L.sb_d) : nullptr, reinterpret_cast<float*>(S + L.st_d));
    gv_prefix_inline(d);
    rc = gv_launch_matmul(d, K, cb, batch, 0, true, st);
    if (rc != kOk) return rc;
    return dec_finish(d, x, cb, h, h_stride, ss_out, y_out, y_stride, peers, batch, hidden, st, fold_out);
}

extern "C" int exl3b200_decode_mlp(int batch, int hidden, int inter, int K, int cb, float* h, long long h_stride,
                                   const float* ss_in, float* ss_out, const void* norm_w, float eps,
                                   const exl3b200_linear* gate, const exl3b200_linear* up,
                                   const exl3b200_linear* down, float swiglu_limit, float* y_out, long long y_stride,
                                   const exl3b200_peers* peers, void* state, size_t state_bytes, void* scratch,
                                   size_t scratch_bytes, void* stream)
{
    return dec_mlp(batch, hidden, inter, K, cb, h, h_stride, ss_in, ss_out, norm_w, eps, gate, up, down,
                   swiglu_limit, y_out, y_stride, peers, state, state_bytes, scratch, scratch_bytes, stream);
}

extern "C" int exl3b200_residual_add(int batch, int hidden, float* h, long long h_stride, const float* y,
                                     long long y_stride, float* ss_out, void* stream)
{
    if (!h || !y || !ss_out) return kErrNullPointer;
    if (batch < 1 || hidden <= 0 || hidden % 128 || h_stride < hidden || y_stride < hidden) return kErrBadShape;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    return dec_launch(exl3_dec_residual_kernel, dec_grid(batch * (hidden / 128)), 256, st, h, h_stride, y, y_stride,
                      ss_out, batch, hidden);
}

extern "C" int exl3b200_decode_layer_workspace(int rows, int hidden, int q_heads, int kv_heads, int inter, int max_ctx,
                                               size_t* state_bytes, size_t* scratch_bytes)
{
    if (!state_bytes || !scratch_bytes) return kErrNullPointer;
    if (rows < 1 || rows > EXL3B200_GEMV_MAX_M || hidden <= 0 || hidden % 128 || q_heads < 1 || kv_heads < 1 ||
        q_heads % kv_heads || q_heads / kv_heads > kAttnMaxGroup || max_ctx < 1 || inter <= 0 || inter % 128)
        return kErrBadShape;
    const DecLayerLayout L = dec_layer_layout(rows, hidden, q_heads, kv_heads, inter, max_ctx);
    *state_bytes = L.state_bytes;
    *scratch_bytes = L.scratch_bytes;
    return kOk;
}

// One decoder layer (attention sub-layer, then MLP sub-layer) with the RMSNorm input
// stages folded into the residual epilogues: the attention's residual epilogue writes
// the MLP's gate/up inputs, the MLP's writes the next layer's q/k/v inputs (when next
// is given), and the consumers (SwiGLU, RoPE) apply the rows' exact norm factors.
extern "C" int exl3b200_decode_layer_step(int rows, int rows_per_seq, int hidden, int q_heads, int kv_heads, int inter,
                                          int K, int cb, float* h, long long h_stride, float* ss_a, float* ss_b,
                                          float eps, const exl3b200_decode_layer* layer,
                                          const exl3b200_decode_layer* next, int input_ready, void* k_cache,
                                          void* v_cache, int max_ctx, const long long* pos, const float* inv_freq,
                                          float swiglu_limit, const exl3b200_peers* peers, void* state,
                                          size_t state_bytes, void* scratch, size_t scratch_bytes, void* stream)
{
    if (!layer || !ss_a || !ss_b || !state || !scratch) return kErrNullPointer;
    if (!layer->attn_norm_w || !layer->mlp_norm_w) return kErrNullPointer;
    size_t need_state = 0, need_scratch = 0;
    int rc = exl3b200_decode_layer_workspace(rows, hidden, q_heads, kv_heads, inter, max_ctx, &need_state,
                                             &need_scratch);
    if (rc != kOk) return rc;
    if (state_bytes < need_state || scratch_bytes < need_scratch) return kErrWorkspace;
    if (((uintptr_t) state & 255) || ((uintptr_t) scratch & 255)) return kErrUnaligned;
    const int nq = q_heads * kHeadDim, nkv = kv_heads * kHeadDim;
    if (!dec_linear_ok(layer->gate, hidden, inter) || !dec_linear_ok(layer->up, hidden, inter)) return kErrBadShape;
    if (next && (!next->attn_norm_w || !dec_linear_ok(next->q, hidden, nq) || !dec_linear_ok(next->k, hidden, nkv) ||
                 !dec_linear_ok(next->v, hidden, nkv)))
        return next->attn_norm_w ? kErrBadShape : kErrNullPointer;
    const DecLayerLayout L = dec_layer_layout(rows, hidden, q_heads, kv_heads, inter, max_ctx);
    char* S = reinterpret_cast<char*>(state);
    char* W = reinterpret_cast<char*>(scratch);
    char* WM = W + L.A.scratch_bytes;
    float* fold_c = reinterpret_cast<float*>(W + L.fold_c);
    const bool mul1 = cb == 2;
    auto target = [&](char* base, size_t xd, size_t sb, const exl3b200_linear* l) {
        return FoldTarget{reinterpret_cast<uint32_t*>(base + xd), mul1 ? reinterpret_cast<float*>(base + sb) : nullptr,
                          reinterpret_cast<const __half*>(l->suh), hidden};
    };
    DecFoldOut fa = {};  // attention residual -> this layer's gate/up inputs
    fa.n = 2;
    fa.t[0] = target(WM, L.M.xd_g, L.M.sb_g, layer->gate);
    fa.t[1] = target(WM, L.M.xd_u, L.M.sb_u, layer->up);
    fa.norm_w = layer->mlp_norm_w;
    fa.fold_c = fold_c;
    DecFoldOut fm = {};  // MLP residual -> the next layer's q/k/v inputs
    if (next) {
        fm.n = 3;
        fm.t[0] = target(W, L.A.xd_q, L.A.sb_q, next->q);
        fm.t[1] = target(W, L.A.xd_k, L.A.sb_k, next->k);
        fm.t[2] = target(W, L.A.xd_v, L.A.sb_v, next->v);
        fm.norm_w = next->attn_norm_w;
        fm.fold_c = fold_c;
    }
    rc = dec_attention(rows, rows_per_seq, hidden, q_heads, kv_heads, K, cb, h, h_stride, ss_a, ss_b,
                       layer->attn_norm_w, eps, layer->q, layer->k, layer->v, layer->o, k_cache, v_cache, max_ctx, pos,
                       inv_freq, nullptr, 0, peers, S, L.A.state_bytes, W, L.A.scratch_bytes, stream,
                       input_ready ? fold_c : nullptr, &fa);
    if (rc != kOk) return rc;
    return dec_mlp(rows, hidden, inter, K, cb, h, h_stride, ss_b, ss_a, layer->mlp_norm_w, eps, layer->gate, layer->up,
                   layer->down, swiglu_limit, nullptr, 0, peers, S + L.A.state_bytes, L.M.state_bytes, WM,
                   L.M.scratch_bytes, stream, fold_c, next ? &fm : nullptr);
}
