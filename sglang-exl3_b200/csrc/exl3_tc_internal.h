// Internal interface of the grouped tensor-core matmul (exl3_tc.cu) for the
// routed-MoE pipeline (exl3_tc_moe.cu): a launch over many problems that share k,
// n, K and the codebook, each with its own trellis, svh, rows and output, whose
// tiles and problem table were written on the device by an earlier kernel.
#pragma once

#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace exl3b200 {

// One problem of a grouped launch (written by a routing kernel).
struct TcProblem {
    const uint8_t* xt;       // input image holding the problem's rows (layout below)
    const uint8_t* trellis;  // [k/16][n/16][32K bytes]
    const __half* svh;       // [n]
    float* out;              // grouped store: fp32 output of the problem's row 0
    int m;                   // rows
    int mtiles;              // ceil(m / 256)
    int tile_begin;          // first tile of the problem in the launch's tile list
    int row0;                // first row in the input image (multiple of 8)
    int slot0;               // first routed slot (token / weight lists) of the problem
    int pad;
    const __half* suh2;      // fused gate|up (kTcGroupedSwiglu, gate problem): down projection suh
};

enum TcMode : int {
    kTcDense = 0,         // one problem, host-known sizes (exl3b200_gemm)
    kTcGroupedStore = 1,  // fp32 out rows of each problem (whole tiles stored, split tiles added)
    kTcGroupedCombine = 2, // fp32 out[slot_token[s]] += slot_weight[s] * y
    kTcDenseSwiglu = 3,    // one fused gate|up problem; a tile is 128 gate + the matching 128 up
                           // columns, its epilogue writes the down projection's rotated input image
    kTcGroupedSwiglu = 4   // routed experts: problem p (gate) and p + 1 (up) of the table form one
                           // problem; a tile is 128 rows x (gate block j | up block j), each half
                           // with its own input image, whole tiles only; the epilogue writes the
                           // down projection's input image at the expert's rows
};

// Rows per kTcGroupedSwiglu tile: A rows 32..127, i.e. TMEM lanes 32..127 (quarters 1..3),
// so that a tile of at most 32 rows is finished by the warps of lane quarter 1 alone.
constexpr int kTcSwRows = 96;

// Input image of a grouped launch: k-chunk major, xt_rows rows of 128 bytes per
// 64-wide k chunk, each 8-row group's 16-byte chunks XOR-swizzled by (row % 8):
// byte ((kc * xt_rows + row) * 128 + ((((kk & 63) >> 3) ^ (row & 7)) << 4) + (kk & 7) * 2)
// holds element kk of row row.  A problem's rows start at a multiple of 8.
__host__ __device__ __forceinline__ size_t tc_image_offset(long long xt_rows, int row, int kk)
{
    return ((size_t) (kk >> 6) * (size_t) xt_rows + (size_t) row) * 128 + (size_t) ((((kk & 63) >> 3) ^ (row & 7)) << 4) +
           (size_t) (kk & 7) * 2;
}

struct TcGroupedCall {
    long long xt_rows;        // rows of every problem's input image
    const TcProblem* probs;
    const int* tile_prob;     // problem index of every tile of the list
    const int* dev_tiles;     // device: number of tiles of this launch
    const int* dev_tile_base; // device: first tile of this launch in the list (nullable: 0)
    int k, n;
    float* out;               // combine: fp32 [tokens][n]
    long long out_stride;     // elements, multiple of 4 (both modes)
    const int* slot_token;    // combine
    const float* slot_weight; // combine
    int mode;                 // kTcGroupedStore, kTcGroupedCombine or kTcGroupedSwiglu
    uint8_t* img;             // swiglu: the down projection's input image (xt_rows rows, k = n)
    float swiglu_limit;       // swiglu: 0 or infinite = no clip
};

// Enqueues one grouped launch (programmatic dependent of the previous kernel).
int tc_grouped_matmul(const TcGroupedCall& c, int K, int cb, cudaStream_t stream);

// SMs of the current device.
int tc_device_sms();

// One dense tensor-core matmul launch sequence (exl3_tc.cu).  img == null: plain
// epilogue into out; img != null: n = 2 * inter fused gate|up columns, the SwiGLU
// epilogue writes the down projection's input image (k = inter) into img.
struct TcDenseRun {
    const void* x;          // input rows (run_input)
    long long x_stride;
    const __half* suh;      // null: x already rotated
    bool run_input;         // false: xt was written by an earlier kernel
    uint8_t* xt;            // input image, tc_xt_bytes(m, k)
    const void* trellis;
    const __half* svh;
    int m, k, n, K, cb;
    void* out;
    long long out_stride;
    int out_dtype;
    uint8_t* img;           // swiglu: output image, tc_xt_bytes(m, n / 2)
    const __half* suh2;     // swiglu: down projection suh [n / 2]
    float swiglu_limit;
    float* slots;           // tc_state_bytes(), zeroed, left zeroed
    int pair = -1;          // CTA-pair tiles: -1 from kTcPairMinRows rows, 0 never, 1 always
};

// When a dense launch uses the CTA-pair kernel (512-row tiles), from measured crossovers
// on one B200 (CUDA-graph replays, weights above L2): the fused SwiGLU gate|up (config 2
// block: 1.891 -> 1.661 ms at 2048 rows, equal at 512) from 512 rows; plain GEMMs only
// from 2048 rows with k >= 16384 (25600 -> 5120 K=4: 606 -> 570 us; but 8192 -> 28672
// K=4: 985 -> 1040 us, and 768 rows lose everywhere to half-empty pair tiles).
constexpr int kTcPairMinRows = 512;
constexpr int kTcPairDenseMinRows = 2048;
constexpr int kTcPairDenseMinK = 16384;
int tc_dense_run(const TcDenseRun& r, cudaStream_t stream);
size_t tc_xt_bytes(int m, int k);
size_t tc_state_bytes();

}  // namespace exl3b200
