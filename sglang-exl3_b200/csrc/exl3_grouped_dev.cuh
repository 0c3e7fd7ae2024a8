// Device-side helpers of the grouped small-M matmul shared by its kernels
// (exl3_gemv.cu) and the fused decode-layer kernels (exl3_decode.cu): problem
// lookup in a launch's table, task-to-problem search, and the epilogue's finish
// of one (problem, 128-column block, row): read and re-zero the summed partials,
// mul1 correction, H128, svh / sqrt(128).
#pragma once

#include "exl3_common.cuh"
#include "exl3_grouped.cuh"

namespace exl3b200 {

__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ const GvProblem& gv_prob(const GvArgs& a, int i)
{
    const int j = i * a.stride + a.offset;
    return a.dev ? a.dev[j] : a.inl[j];
}

struct GvTotals {
    int nprob, units, in_tasks, out_tasks;
};

__device__ __forceinline__ GvTotals gv_totals(const GvArgs& a)
{
    GvTotals t;
    if (a.dev_totals) {
        t.nprob = __ldcg(a.dev_totals + 0);
        t.units = __ldcg(a.dev_totals + 1);
        t.in_tasks = __ldcg(a.dev_totals + 2);
        t.out_tasks = __ldcg(a.dev_totals + 3);
    } else {
        t.nprob = a.nprob;
        t.units = a.units;
        t.in_tasks = a.in_tasks;
        t.out_tasks = a.out_tasks;
    }
    if (a.uniform_units > 0) t.units = t.nprob * a.uniform_units;
    return t;
}

// largest problem index whose task range starts at or before task
template <int WHICH>
__device__ __forceinline__ int gv_find(const GvArgs& a, int nprob, int task)
{
    int lo = 0, hi = nprob - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        const GvProblem& p = gv_prob(a, mid);
        const int begin = WHICH == 0 ? p.in_task_begin : WHICH == 1 ? p.out_task_begin : p.unit_begin;
        if (begin <= task) lo = mid;
        else hi = mid - 1;
    }
    return lo;
}

// The block-row's output scales (loaded ahead of the partial sums, so the two
// memory round trips overlap).
__device__ __forceinline__ void gv_load_svh(const GvProblem& p, int nb, int lane, float (&sv)[4])
{
#pragma unroll
    for (int e = 0; e < 4; ++e) sv[e] = __half2float(p.svh[nb * 128 + lane + 32 * e]);
}

// Summed partials of one (problem, block, row) -> outputs: mul1 correction, H128,
// * 1/sqrt(128) * svh.  Lane holds columns lane + 32 e.
template <int CB>
__device__ __forceinline__ void gv_finish_math(const GvProblem& p, int r, int lane, const float (&sv)[4], float (&v)[4])
{
    if constexpr (CB == 2) {
        const float k_inv = __half2float(__ushort_as_half(kMul1InvBits));
        const float k_bias = __half2float(__ushort_as_half(kMul1BiasBits));
        const int nblk = p.k >> 7;
        float sum = 0.f;
        for (int b = lane; b < nblk; b += 32) sum += __ldcg(p.sblk + (size_t) r * nblk + b);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
#pragma unroll
        for (int e = 0; e < 4; ++e) v[e] = fmaf(k_inv, v[e], k_bias * sum);
    }
    warp_fwht128(v, lane);
#pragma unroll
    for (int e = 0; e < 4; ++e) v[e] = v[e] * kHadScale * sv[e];
}

// Read and re-zero the split-K partials of (problem, block nb, row r) in the state,
// then finish them.
template <int CB>
__device__ __forceinline__ void gv_finish(const GvProblem& p, int nb, int r, int lane, float (&v)[4])
{
    float sv[4];
    gv_load_svh(p, nb, lane, sv);
    float* src = p.acc + (size_t) nb * p.acc_nb_stride + (size_t) r * 128;
#pragma unroll
    for (int e = 0; e < 4; ++e) v[e] = __ldcg(src + lane + 32 * e);
#pragma unroll
    for (int e = 0; e < 4; ++e) __stcg(src + lane + 32 * e, 0.f);
    gv_finish_math<CB>(p, r, lane, sv, v);
}

// Bring 256 bytes of constant data (scales, norm weights) into L2; safe before the
// previous kernel in the stream has finished.
__device__ __forceinline__ void prefetch_l2_256(const void* ptr, int lane)
{
    if (lane < 2) asm volatile("prefetch.global.L2 [%0];" ::"l"(reinterpret_cast<const char*>(ptr) + 128 * lane));
}

// Before griddep_wait: prefetch the output scales of the warp's first epilogue task
// (host-built tables only: a device table may still be in the making).
__device__ __forceinline__ void gv_prefetch_epilogue(const GvArgs& a, int lane)
{
    if (a.dev || a.dev_totals) return;
    const int task = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (task >= a.out_tasks) return;
    const GvProblem& p = gv_prob(a, gv_find<1>(a, a.nprob, task));
    prefetch_l2_256(p.svh + (size_t) ((task - p.out_task_begin) % (p.n >> 7)) * 128, lane);
}

}  // namespace exl3b200
