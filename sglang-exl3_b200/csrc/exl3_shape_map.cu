// Kernel-shape map of the B200 backend: which kernel family serves a problem.
//
// The reference declares select_gemm_shape(cc, m, k, n, bits, multi) and a
// compatibility test per shape (csrc/quant/exl3_kernel_map.cuh:3-12); its table of
// mma.sync tile shapes (16 rows x 128..512 columns) lives in the unvendored
// exllamav3.  Here the families are the small-M register-decode kernel (two row
// groupings, two tilings), the tcgen05 kernel and the two routed-MoE pipelines, and
// the table holds the row counts at which one family overtakes another, per K.
//
// Crossovers, measured on one B200 (CUDA-graph replays of rotating weight copies,
// small-M in 16-row chunks against the tensor-core kernel):
// * dense: 16 rows - small-M wins at every shape and K tried (8192x8192,
//   8192x28672, 5120x25600, 25600x5120, 2048x1024, 8192x1024; K 2, 3, 4; e.g.
//   8192x28672 K=4: 94.9 us vs 117.5 us); 24 rows - the tensor-core kernel wins
//   everywhere (153.8 us vs 121.2 us), and from there on the gap widens (96 rows:
//   565.5 vs 152.3 us).  So the tensor-core kernel takes 17 rows and more - for large
//   matrices.  Up to 2^24 weights (2048x2048, 1024x2048, 4096x1536 K=3, 8192x1024,
//   2048x8192; us per launch, 16-row chunks / tensor cores, later kernels) two chunks
//   still win at 32 rows (e.g. 8192x1024 K=4: 21.5 / 23.3; 4096x1536 K=3: 22.4 / 27.3)
//   and lose from 48 (32.6 / 24.2; 33.4 / 28.1): the tensor cores from 33 rows there.
// * the 4-tiles-per-warp tiling at 3 CTAs per SM was slower than 8 tiles at 2 CTAs
//   at every M=1 shape measured (TP8 shards to the full 70B gate/up; K 3 and 4), so
//   the map never selects it (it stays reachable through the flags for tests).
// * inside the tcgen05 family the dense launch takes CTA-pair tiles (512 x 256 over a
//   2-CTA cluster) for the fused SwiGLU gate|up from 512 rows and for plain GEMMs from
//   2048 rows with k >= 16384 (kTcPairMinRows / kTcPairDenseMinRows / kTcPairDenseMinK,
//   exl3_tc_internal.h, with the measurements).
// * routed MoE: the tensor-core pipeline wins from 10-14 average rows per local
//   expert (config 5 at 7.5 rows: small-M 1.11 vs 1.32 ms; 10 rows: 1.20 vs 1.34;
//   config 3 at 14 rows: 1.29 vs 1.52; config 5 at 20 rows: 1.37 vs 2.10), hence 12.
#include "exl3_capi_internal.h"

namespace exl3b200 {

struct ShapeRule {
    int K;
    int gv8_max_rows;       // small-M with one 8-row group up to here, then two 8-row groups
    int tc_min_rows;        // tensor-core kernel from here (below: 16-row small-M chunks)
    int tc_min_rows_small;  // the same for matrices of at most kSmallWeights weights
    int moe_tc_rows;        // routed MoE: tensor-core pipeline from this many rows per expert
};

constexpr ShapeRule kShapeRules[] = {
    {2, 8, 17, 33, 12},
    {3, 8, 17, 33, 12},
    {4, 8, 17, 33, 12},
};

// Below this many weights (k x n) a tensor-core launch has few 256 x 256 tiles and two
// 16-row small-M chunks stay faster up to 32 rows.
constexpr long long kSmallWeights = 1ll << 24;

constexpr exl3b200_shape_desc kShapes[] = {
    {"none", 0, 0, 0, 0},
    {"small-M 8 rows, 8 tiles/warp, 2 CTAs/SM", 8, 8, 128, 2},
    {"small-M 8 rows, 4 tiles/warp, 3 CTAs/SM", 8, 8, 128, 3},
    {"small-M 16 rows, 4 tiles/warp, 2 CTAs/SM", 16, 16, 128, 2},
    {"tcgen05 256x256 persistent", 0, 256, 256, 1},
    {"routed MoE, small-M pipeline", 16, 16, 128, 2},
    {"routed MoE, grouped tcgen05", 0, 256, 256, 1},
};
constexpr int kNumShapes = (int) (sizeof(kShapes) / sizeof(kShapes[0])) - 1;

static const ShapeRule* rule_for(int K)
{
    for (const ShapeRule& r : kShapeRules)
        if (r.K == K) return &r;
    return nullptr;
}

}  // namespace exl3b200

using namespace exl3b200;

extern "C" int exl3b200_num_shapes(void) { return kNumShapes; }

extern "C" int exl3b200_shape_compat(int shape, int m, int k, int n, int K)
{
    if (shape < 1 || shape > kNumShapes || m < 1 || K < 2 || K > 4) return 0;
    if (k <= 0 || n <= 0 || k % 128 || n % 128) return 0;
    const int max_rows = kShapes[shape].max_rows;
    return (max_rows == 0 || m <= max_rows) ? 1 : 0;
}

extern "C" int exl3b200_select_shape(int m, int k, int n, int K, int cb, int experts, int topk)
{
    if (cb < 0 || cb > 2 || m < 1) return 0;
    const ShapeRule* r = rule_for(K);
    if (!r) return 0;
    if (experts > 0) {
        const long long pairs = (long long) m * (topk > 0 ? topk : 1);
        return pairs >= (long long) r->moe_tc_rows * experts ? EXL3B200_SHAPE_MOE_TC : EXL3B200_SHAPE_MOE_SMALL;
    }
    if (m <= r->gv8_max_rows) return EXL3B200_SHAPE_GV8;
    const bool small = (long long) k * n <= kSmallWeights;
    if (m < (small ? r->tc_min_rows_small : r->tc_min_rows)) return EXL3B200_SHAPE_GV16;
    return EXL3B200_SHAPE_TC;
}

extern "C" int exl3b200_shape_info(int shape, exl3b200_shape_desc* out)
{
    if (!out) return EXL3B200_ENULL;
    if (shape < 1 || shape > kNumShapes) return EXL3B200_EBADARG;
    *out = kShapes[shape];
    return EXL3B200_OK;
}
