// Grouped small-M EXL3 matmul: shared declarations.
//
// A launch works on a table of problems.  Each problem is one EXL3 linear
// (trellis, suh, svh) applied to m <= 16 input rows that may be gathered from a
// larger activation matrix, with its own rotated-input scratch, partial-sum
// state and output.  All problems of a launch share K (bits) and the codebook.
//
// The table is either inline in the kernel parameters (host-built, up to
// kGvInline problems: fused q/k/v, gate/up, a single linear) or in device memory
// (built on the device from routing data: batched experts, routed MoE), in which
// case the problem count and the task totals are read from device memory, so no
// host synchronisation is ever needed.
#pragma once

#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace exl3b200 {

constexpr int kGvInline = 8;
constexpr int kGvMaxRows = 16;

// epilogue modes
enum GvEpilogue : int {
    kEpiStore = 0,    // out[r * out_stride + col] = y (out dtype)
    kEpiCombine = 1,  // fp32 out[out_rows[r] * out_stride + col] += out_scale[r] * y (atomic)
    kEpiSwiglu = 2,   // problems (2q, 2q+1) = (gate, up); writes the rotated down-projection
                      // input: out (uint32 dup pairs) [r][col], pre-scale out_suh
    kEpiSwigluFused = 3,  // one fused gate|up problem (n = 2 * inter): block nb pairs with block
                          // nb + n / 256; output as kEpiSwiglu; out_tasks = m * n / 256
};

struct GvProblem {
    const uint32_t* trellis;  // [k/16][n/16][16K] as uint32 words
    const __half* suh;        // [k] input sign/scale (null: input already rotated, plain copy)
    const __half* svh;        // [n]
    const __half* x;          // input rows (fp16)
    const int* x_rows;        // input row of problem row r (null: r)
    uint32_t* xd;             // [m][k] rotated input as duplicated fp16 pairs
    float* sblk;              // [m][k/128] block sums of the rotated input (mul1 only, else null)
    float* acc;               // zeroed partial sums: block nb, row r at acc[nb*acc_nb_stride + r*128]
    void* out;                // output (see epilogue modes)
    const int* out_rows;      // combine: output row of problem row r
    const float* out_scale;   // combine: weight of problem row r
    const __half* out_suh;    // swiglu: down-projection input sign/scale [n]
    float* out_sblk;          // swiglu, mul1 down projection: block sums of the written input
    long long x_stride;
    long long out_stride;
    int k, n, m;
    int acc_nb_stride;        // floats between consecutive 128-column blocks of acc
    int unit_begin;           // first matmul unit (tables with per-problem shapes)
    int in_task_begin;        // first input-stage task (warp task = row x 128-block)
    int out_task_begin;       // first epilogue task
};

// Launch-wide view of a table.
struct GvArgs {
    GvProblem inl[kGvInline];
    const GvProblem* dev;     // device table (used instead of inl when non-null)
    const int* dev_totals;    // device [nprob, units, in_tasks, out_tasks] (null: host values)
    int nprob, units, in_tasks, out_tasks;
    int stride, offset;       // problem i of this launch is table entry i*stride + offset
    int uniform_units;        // > 0: every problem has this many units (unit_begin unused)
    int cta_per_block;        // > 0: matmul CTAs per 128-column block (block-aligned split; set by the launcher)
    int block_units;          // k-slices of every block when cta_per_block > 0
    int out_dtype;            // 0 fp16, 1 bf16, 2 fp32 (store mode)
    int epi_mode;
    float swiglu_limit;       // swiglu: 0 or infinite = no clip
};

// Host launchers (exl3_gemv.cu).  Grid sizes are fixed upper bounds; with device
// totals every kernel reads the real extent and idles the rest.
int gv_launch_input(const GvArgs& a, int max_in_tasks, bool pdl, cudaStream_t stream);
int gv_launch_matmul(const GvArgs& a, int K, int cb, int max_rows, int variant, bool pdl, cudaStream_t stream);
int gv_launch_epilogue(const GvArgs& a, int cb, int max_out_tasks, bool pdl, cudaStream_t stream);

// Fill the task prefixes of an inline (host-built) table.
void gv_prefix_inline(GvArgs& a);

size_t gv_state_bytes_per_problem(int n);
size_t gv_xd_bytes(int m, int k);
size_t gv_sblk_bytes(int m, int k);
int gv_sm_count();

}  // namespace exl3b200
