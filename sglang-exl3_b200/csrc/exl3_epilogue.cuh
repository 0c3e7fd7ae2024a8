// Epilogue of one (problem, 128-column block, row) of the grouped small-M matmul,
// shared by the epilogue kernels of exl3_gemv.cu and exl3_decode.cu: read and
// re-zero the block's summed partials (gv_finish), then one of
//   kEpiStore     out = y (fp16 / bf16 / fp32)
//   kEpiCombine   fp32 out[out_rows[r]] += out_scale[r] * y (routed MoE combine)
//   kEpiSwiglu    (gate, up) pair -> clipped SwiGLU -> the down projection's rotated
//                 input (csrc/quant/hadamard_inner.cuh:283-413, csrc/p2b_moe.cu:300-336
//                 of the reference)
//   kEpiRopeKV    decode q/k/v: RoPE (rotate-half), q scaled into the attention
//                 buffer, k and v appended to the bf16 cache
//   kEpiResidual  decode: h += y and the row's sum of squares (with the norm fold,
//                 also the next sub-layer's normalised, rotated inputs)
#pragma once

#include <cuda_bf16.h>

#include "exl3_common.cuh"
#include "exl3_grouped.cuh"
#include "exl3_grouped_dev.cuh"

namespace exl3b200 {

constexpr int kHeadDim = 128;

enum DecEpiMode : int { kEpiRopeKV = 10, kEpiResidual = 11 };

// peer buffer: [control 256 B: PeerCtl at 0, generation word at kPeerGen]
//              [data: 2 parities x 8 ranks x max_rows x hidden 8-byte slots]
// A slot holds one fp32 partial and the tag of the call that wrote it in one
// 8-byte store, so a reader that sees the tag sees the value (no fence, no counter).
constexpr int kPeerMaxRanks = 8;
constexpr size_t kPeerGen = 64;    // u32: generation, advanced by every exl3b200_peer_reset
constexpr size_t kPeerData = 256;
constexpr unsigned long long kPeerTimeoutNs = 2000000000ull;

struct PeerCtl {
    unsigned int epoch;     // calls completed
    unsigned int done;      // CTAs of the running reduce that finished
    unsigned int poisoned;  // a wait gave up: exchanges return at once until the host re-arms
};

// One input of the next sub-layer that a residual epilogue writes itself (norm fold):
// the rotated-input image (duplicated fp16 pairs) and, for mul1, its block sums.
struct FoldTarget {
    uint32_t* xd;        // [rows][k]
    float* sblk;         // [rows][k/128] or null
    const __half* suh;   // [k]
    int k;
};

constexpr int kFoldMax = 3;
// The folded input is fp16(h * c * w) with c = rsqrt(ss_old/hidden + eps) / 16 (ss_old:
// the row's sum of squares before the residual add, known while the add runs); the
// consumer multiplies its finished outputs by rsqrt(ss_new/hidden + eps) / c.  The
// power-of-two factor keeps 16x headroom below the fp16 range for rows whose norm
// grows across the add, and is exact.
constexpr float kFoldHeadroom = 0.0625f;

struct DecAux {
    // norm input stage
    const float* h;
    long long h_stride;
    const float* ss_in;
    float* ss_out;           // zeroed by the norm input stage (rows zero_rows)
    int zero_rows;
    const __nv_bfloat16* norm_w;
    float eps;
    float inv_hidden;
    // RoPE / KV append / attention
    const long long* pos;    // position of the new token (= tokens already cached)
    const float* inv_freq;   // [head_dim / 2]
    float* qbuf;             // [batch][q_heads][128], scaled by 1/sqrt(128)
    __nv_bfloat16* k_cache;  // [batch][kv_heads][max_ctx][128]
    __nv_bfloat16* v_cache;
    long long cache_b_stride, cache_h_stride;
    int max_ctx, q_heads, kv_heads;
    int rows_per_seq;        // rows r = R s + j (j < R) are sequence s at position *pos + j
    // residual epilogue
    float* resid;
    long long resid_stride;
    float* ss_acc;
    // norm fold, output side (residual epilogues): write the next sub-layer's inputs
    int fold_n;                          // 0: off
    FoldTarget fold[kFoldMax];
    const __nv_bfloat16* fold_norm_w;    // the next sub-layer's RMSNorm weight
    float* fold_c;                       // [rows]: the pre-scale c written for the consumer
    // norm fold, input side (RoPE / SwiGLU epilogue): finished values *=
    // rsqrt(ss_in/hidden + eps) / fold_c_in[r]; the consumer also zeroes zero_ss
    const float* fold_c_in;
    float* zero_ss;
    // tensor-parallel partial exchange
    char* peer[kPeerMaxRanks];
    int peer_world, peer_rank, peer_rows, peer_hidden;
    unsigned long long peer_wait_ns;  // limit of the arrival wait
    int* status;
};

// Slots of row `row` written by rank `src` in rank q's buffer (hidden slots).
__device__ __forceinline__ unsigned long long* peer_slot(const DecAux& x, int q, unsigned int parity, int src, int row)
{
    return reinterpret_cast<unsigned long long*>(x.peer[q] + kPeerData) +
           (((size_t) parity * kPeerMaxRanks + src) * x.peer_rows + row) * x.peer_hidden;
}

__device__ __forceinline__ void st_slot_sys(unsigned long long* p, float v, unsigned int tag)
{
    const unsigned long long w = ((unsigned long long) tag << 32) | __float_as_uint(v);
    asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}

__device__ __forceinline__ unsigned long long ld_slot_sys(const unsigned long long* p)
{
    unsigned long long w;
    asm volatile("ld.relaxed.sys.global.b64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    return w;
}

__device__ __forceinline__ unsigned long long globaltimer_ns()
{
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ unsigned int ld_acquire_sys(const unsigned int* p)
{
    unsigned int v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void st_release_sys(unsigned int* p, unsigned int v)
{
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// fp16 values (already rounded) of one 128-block -> a problem's rotated input
// (the GEMV input stage's layout: fp16 x*suh, H128, /sqrt(128) as duplicated fp16
// pairs; block sums for mul1).
// The input scales of one 128-block (suh[b * 128 + lane + 32 i]) are passed loaded.
__device__ __forceinline__ void store_rotated_s(uint32_t* xd, float* sblk, bool rotate, const float (&su)[4], int k,
                                                int r, int b, int lane, const float (&xv)[4])
{
    float v[4];
    if (rotate) {
#pragma unroll
        for (int i = 0; i < 4; ++i) v[i] = __half2float(__float2half_rn(__fmul_rn(xv[i], su[i])));
        warp_fwht128(v, lane);
#pragma unroll
        for (int i = 0; i < 4; ++i) v[i] = __fmul_rn(v[i], kHadScale);
    } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) v[i] = xv[i];
    }
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const __half hh = __float2half_rn(v[i]);
        const uint32_t u = __half_as_ushort(hh);
        xd[(size_t) r * k + b * 128 + lane + 32 * i] = u | (u << 16);
        s += __half2float(hh);
    }
    if (sblk) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        if (lane == 0) sblk[(size_t) r * (k >> 7) + b] = s;
    }
}

__device__ __forceinline__ void store_rotated(uint32_t* xd, float* sblk, const __half* suh, int k, int r, int b,
                                              int lane, const float (&xv)[4])
{
    float su[4] = {1.f, 1.f, 1.f, 1.f};
    if (suh) {
#pragma unroll
        for (int i = 0; i < 4; ++i) su[i] = __half2float(suh[b * 128 + lane + 32 * i]);
    }
    store_rotated_s(xd, sblk, suh != nullptr, su, k, r, b, lane, xv);
}

// Norm fold, output side.  Everything a residual epilogue task needs besides the new
// row values, loaded at the task's start so the loads overlap the partial sums' read:
// the pre-scale c (from the row's sum of squares before the add), the next
// sub-layer's norm weights and every target's input scales of block nb.
struct FoldPre {
    float c;
    float w[4];
    float su[kFoldMax][4];
};

__device__ __forceinline__ void fold_preload(const DecAux& x, int r, int nb, int lane, FoldPre& f)
{
    f.c = rsqrtf(x.ss_in[r] * x.inv_hidden + x.eps) * kFoldHeadroom;
#pragma unroll
    for (int e = 0; e < 4; ++e) f.w[e] = __bfloat162float(x.fold_norm_w[nb * 128 + lane + 32 * e]);
#pragma unroll
    for (int i = 0; i < kFoldMax; ++i)
#pragma unroll
        for (int e = 0; e < 4; ++e)
            f.su[i][e] = i < x.fold_n ? __half2float(x.fold[i].suh[nb * 128 + lane + 32 * e]) : 0.f;
}

// Before a residual epilogue's dependency wait: its first task's fold inputs into L2.
__device__ __forceinline__ void fold_prefetch(const DecAux& x, int nb, int lane)
{
    prefetch_l2_256(x.fold_norm_w + nb * 128, lane);
    for (int i = 0; i < x.fold_n; ++i) prefetch_l2_256(x.fold[i].suh + nb * 128, lane);
}

// Block nb of row r of the new residual stream (nv) -> the next sub-layer's rotated
// inputs, pre-scaled by c (see kFoldHeadroom).
__device__ __forceinline__ void fold_out(const DecAux& x, int r, int nb, int lane, const float (&nv)[4],
                                         const FoldPre& f)
{
    float xv[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) xv[e] = __half2float(__float2half_rn(nv[e] * f.c * f.w[e]));
#pragma unroll
    for (int i = 0; i < kFoldMax; ++i) {
        if (i < x.fold_n) {
            const FoldTarget& t = x.fold[i];
            store_rotated_s(t.xd, t.sblk, true, f.su[i], t.k, r, nb, lane, xv);
        }
    }
    if (nb == 0 && lane == 0) x.fold_c[r] = f.c;
}

// Loads and math of an epilogue that do not depend on the partial sums (issued
// first so their round trips overlap the partials' read).
struct EpiPre {
    float pre[4];
    long long pos;
    FoldPre fold;  // residual with the norm fold
};

__device__ __forceinline__ EpiPre epi_preload(const GvProblem& p, const DecAux& x, int mode, int pi, int nb, int r,
                                              int lane)
{
    EpiPre ep;
    float (&pre)[4] = ep.pre;
    long long& pos = ep.pos;
    pos = 0;
#pragma unroll
    for (int e = 0; e < 4; ++e) pre[e] = 0.f;
    if (mode == kEpiSwiglu) {
#pragma unroll
        for (int e = 0; e < 4; ++e) pre[e] = __half2float(p.out_suh[nb * 128 + lane + 32 * e]);
    } else if (mode == kEpiResidual) {
        const float* hr = x.resid + (size_t) r * x.resid_stride + nb * 128;
#pragma unroll
        for (int e = 0; e < 4; ++e) pre[e] = hr[lane + 32 * e];
        if (x.fold_n) fold_preload(x, r, nb, lane, ep.fold);
    } else if (mode == kEpiRopeKV) {
        pos = *x.pos + r % x.rows_per_seq;
        if (pi < 2) {
            const float fpos = (float) pos;
            sincosf(fpos * x.inv_freq[lane], &pre[0], &pre[1]);
            sincosf(fpos * x.inv_freq[lane + 32], &pre[2], &pre[3]);
        }
    }
    return ep;
}

// The output side of an epilogue: v = the finished block row of problem p (for
// SwiGLU the gate), u = the up projection's (SwiGLU only).
template <int CB>
__device__ __forceinline__ void epi_apply(const GvArgs& a, const DecAux& x, int mode, int pi, const GvProblem& p, int nb,
                                          int r, int lane, float (&v)[4], const float (&u)[4], const EpiPre& ep)
{
    const float (&pre)[4] = ep.pre;
    const long long pos = ep.pos;
    if (mode == kEpiStore) {
#pragma unroll
        for (int e = 0; e < 4; ++e)
            store_out(p.out, (size_t) r * p.out_stride + nb * 128 + lane + 32 * e, v[e], a.out_dtype);
    } else if (mode == kEpiCombine) {
        const int orow = p.out_rows ? p.out_rows[r] : r;
        const float w = p.out_scale ? p.out_scale[r] : 1.f;
        float* o = reinterpret_cast<float*>(p.out) + (size_t) orow * p.out_stride + nb * 128;
#pragma unroll
        for (int e = 0; e < 4; ++e) atomicAdd(o + lane + 32 * e, w * v[e]);
    } else if (mode == kEpiSwiglu) {
        const float lim = a.swiglu_limit;
        const bool clip = lim > 0.f && lim < 3.0e38f;
        float act[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            float gv = v[e], uv = u[e];
            if (clip) {
                gv = fminf(gv, lim);
                uv = fminf(fmaxf(uv, -lim), lim);
            }
            const float s = gv / (1.0f + expf(-gv));
            act[e] = __half2float(__float2half_rn(s * uv));
        }
        // rotated input of the down projection for this 128-block of the intermediate
#pragma unroll
        for (int e = 0; e < 4; ++e) act[e] = __half2float(__float2half_rn(__fmul_rn(act[e], pre[e])));
        warp_fwht128(act, lane);
        uint32_t* dst = reinterpret_cast<uint32_t*>(p.out) + (size_t) r * p.out_stride + nb * 128;
        float bsum = 0.f;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const __half hh = __float2half_rn(__fmul_rn(act[e], kHadScale));
            const uint32_t h = __half_as_ushort(hh);
            dst[lane + 32 * e] = h | (h << 16);
            bsum += __half2float(hh);
        }
        if (p.out_sblk) {
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) bsum += __shfl_xor_sync(0xffffffffu, bsum, o);
            if (lane == 0) p.out_sblk[(size_t) r * (p.n >> 7) + nb] = bsum;
        }
    } else if (mode == kEpiRopeKV) {
        // problems 0, 1, 2 = q, k, v; block nb = head nb; lane holds dims lane + 32e;
        // pre = (sin, cos) of the angles of dims lane and lane + 32
        if (pos < 0 || pos >= x.max_ctx) {  // the cache has no row for this position
            if (x.status && lane == 0) atomicCAS(x.status, 0, (int) kErrBadShape);
            return;
        }
        if (pi < 2) {
            const float s0 = pre[0], c0 = pre[1], s1 = pre[2], c1 = pre[3];
            const float n0 = v[0] * c0 - v[2] * s0, n2 = v[2] * c0 + v[0] * s0;
            const float n1 = v[1] * c1 - v[3] * s1, n3 = v[3] * c1 + v[1] * s1;
            v[0] = n0;
            v[1] = n1;
            v[2] = n2;
            v[3] = n3;
        }
        if (pi == 0) {
            float* q = x.qbuf + ((size_t) r * x.q_heads + nb) * kHeadDim;
#pragma unroll
            for (int e = 0; e < 4; ++e) q[lane + 32 * e] = v[e] * kHadScale;  // 1/sqrt(head_dim), head_dim = 128
        } else {
            __nv_bfloat16* c = (pi == 1 ? x.k_cache : x.v_cache) + (size_t) (r / x.rows_per_seq) * x.cache_b_stride +
                               (size_t) nb * x.cache_h_stride + (size_t) pos * kHeadDim;
#pragma unroll
            for (int e = 0; e < 4; ++e) c[lane + 32 * e] = __float2bfloat16_rn(v[e]);
        }
    } else {  // kEpiResidual: pre = h
        float* hr = x.resid + (size_t) r * x.resid_stride + nb * 128;
        float sq = 0.f;
        float nv[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            nv[e] = pre[e] + v[e];
            hr[lane + 32 * e] = nv[e];
            sq += nv[e] * nv[e];
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
        if (lane == 0) atomicAdd(x.ss_acc + r, sq);
        if (x.fold_n) fold_out(x, r, nb, lane, nv, ep.fold);
    }
}

// Norm fold, input side: the factor that turns outputs computed from the pre-scaled
// input into those of the normalised input (1 when the input stage normalised).
__device__ __forceinline__ float fold_factor(const DecAux& x, int r)
{
    return x.fold_c_in ? rsqrtf(x.ss_in[r] * x.inv_hidden + x.eps) / x.fold_c_in[r] : 1.f;
}

template <int CB>
__device__ __forceinline__ void epi_block_row(const GvArgs& a, const DecAux& x, int mode, int pi, const GvProblem& p,
                                              const GvProblem* up, int nb, int r, int lane)
{
    const EpiPre ep = epi_preload(p, x, mode, pi, nb, r, lane);
    const float f = fold_factor(x, r);  // loaded before the partial sums are read and re-zeroed
    float v[4], u[4] = {0.f, 0.f, 0.f, 0.f};
    gv_finish<CB>(p, nb, r, lane, v);
    if (mode == kEpiSwiglu) gv_finish<CB>(*up, nb, r, lane, u);
    if (x.fold_c_in) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            v[e] *= f;
            u[e] *= f;
        }
    }
    epi_apply<CB>(a, x, mode, pi, p, nb, r, lane, v, u, ep);
}

}  // namespace exl3b200
