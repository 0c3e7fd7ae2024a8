// Dense SwiGLU MLP block with the activation fused into the gate|up matmul's
// epilogue: out = down(silu(gate(x)) * up(x)) for a fused gate|up EXL3 trellis (the
// reference's packed13 / "fat GEMM" layout, gate columns then up columns) and an
// EXL3 down projection.
//
// The reference runs the fat GEMM into an fp32 [rows, 2 * inter] buffer, then the
// clip, sigmoid, multiplies and the fp16 copy in torch, then had_r_128 for the down
// projection's input (src/sglang_exl3/exl3.py:1199-1218).  Here the activation and
// the down projection's input transform happen in the gate|up epilogue, which writes
// the down projection's rotated input directly in the layout its matmul reads; no
// [rows, 2 * inter] intermediate exists.  The roundings are the reference's: fp32
// gate/up, fp16 activation, fp16 x * suh, fp32 transform, fp16 result.
//
// Kernel families by the shape map (exl3b200_select_shape on the gate|up problem):
// * small-M (up to 16 rows): one gate|up problem whose epilogue (kEpiSwigluFused)
//   pairs gate block j with up block j and writes the down projection's duplicated
//   fp16 input pairs; the down matmul then runs without an input stage;
// * tensor cores (17 rows and more): the gate|up GEMM's tiles hold gate block j and
//   up block j side by side (kTcDenseSwiglu) and the epilogue writes the down
//   GEMM's shared-memory image; the down GEMM runs without an input stage.
#include "exl3_common.cuh"
#include "exl3_capi_internal.h"
#include "exl3_grouped.cuh"
#include "exl3_tc_internal.h"

namespace exl3b200 {

static size_t align256(size_t v) { return (v + 255) & ~(size_t) 255; }

struct MlpLayout {
    bool tc;
    size_t state, scratch;
    size_t xd_gu, sb_gu, xd_d, sb_d;  // small-M scratch offsets
    size_t st_d;                      // small-M: down projection's state offset
    size_t img1, img2;                // tensor-core scratch offsets
};

static MlpLayout mlp_layout(int m, int hidden, int inter, int K, int cb)
{
    MlpLayout L = {};
    // the small-M path runs one 16-row group: more rows go to the tensor cores
    L.tc = m > EXL3B200_GEMV_MAX_M || exl3b200_select_shape(m, hidden, 2 * inter, K, cb, 0, 0) == EXL3B200_SHAPE_TC;
    if (L.tc) {
        L.state = tc_state_bytes();
        L.img1 = 0;
        L.img2 = align256(tc_xt_bytes(m, hidden));
        L.scratch = L.img2 + align256(tc_xt_bytes(m, inter));
    } else {
        L.st_d = gv_state_bytes_per_problem(2 * inter);
        L.state = L.st_d + gv_state_bytes_per_problem(hidden);
        size_t o = 0;
        L.xd_gu = o; o += gv_xd_bytes(m, hidden);
        L.sb_gu = o; o += gv_sblk_bytes(m, hidden);
        L.xd_d = o; o += gv_xd_bytes(m, inter);
        L.sb_d = o; o += gv_sblk_bytes(m, inter);
        L.scratch = o;
    }
    return L;
}

static int mlp_small(const MlpLayout& L, const exl3b200_mlp_args& p, char* state, char* scratch, cudaStream_t st)
{
    const int m = p.m, H = p.hidden, I = p.inter;
    GvArgs a = {};
    a.nprob = 1;
    a.epi_mode = kEpiSwigluFused;
    a.swiglu_limit = p.swiglu_limit;
    GvProblem& g = a.inl[0];
    g.trellis = reinterpret_cast<const uint32_t*>(p.gate_up.trellis);
    g.suh = reinterpret_cast<const __half*>(p.gate_up.suh);
    g.svh = reinterpret_cast<const __half*>(p.gate_up.svh);
    g.x = reinterpret_cast<const __half*>(p.x);
    g.x_stride = p.x_stride;
    g.xd = reinterpret_cast<uint32_t*>(scratch + L.xd_gu);
    g.sblk = p.cb_gate_up == 2 ? reinterpret_cast<float*>(scratch + L.sb_gu) : nullptr;
    g.acc = reinterpret_cast<float*>(state);
    g.acc_nb_stride = 16 * 128;
    g.out = scratch + L.xd_d;
    g.out_stride = I;  // uint32 pairs per row of the down projection's input
    g.out_suh = reinterpret_cast<const __half*>(p.down.suh);
    g.out_sblk = p.cb_down == 2 ? reinterpret_cast<float*>(scratch + L.sb_d) : nullptr;
    g.k = H;
    g.n = 2 * I;
    g.m = m;
    gv_prefix_inline(a);
    a.out_tasks = m * (I / 128);  // one task per (row, gate/up block pair)
    int rc = gv_launch_input(a, a.in_tasks, false, st);
    if (rc == kOk) rc = gv_launch_matmul(a, p.K_gate_up, p.cb_gate_up, m, 0, true, st);
    if (rc == kOk) rc = gv_launch_epilogue(a, p.cb_gate_up, a.out_tasks, true, st);
    if (rc != kOk) return rc;

    GvArgs b = {};
    b.nprob = 1;
    b.epi_mode = kEpiStore;
    b.out_dtype = p.out_dtype;
    GvProblem& d = b.inl[0];
    d.trellis = reinterpret_cast<const uint32_t*>(p.down.trellis);
    d.svh = reinterpret_cast<const __half*>(p.down.svh);
    d.xd = reinterpret_cast<uint32_t*>(scratch + L.xd_d);
    d.sblk = p.cb_down == 2 ? reinterpret_cast<float*>(scratch + L.sb_d) : nullptr;
    d.acc = reinterpret_cast<float*>(state + L.st_d);
    d.acc_nb_stride = 16 * 128;
    d.out = p.out;
    d.out_stride = p.out_stride;
    d.k = I;
    d.n = H;
    d.m = m;
    gv_prefix_inline(b);
    rc = gv_launch_matmul(b, p.K_down, p.cb_down, m, 0, true, st);  // input written by the epilogue above
    if (rc == kOk) rc = gv_launch_epilogue(b, p.cb_down, b.out_tasks, true, st);
    return rc;
}

static int mlp_tc(const MlpLayout& L, const exl3b200_mlp_args& p, char* state, char* scratch, cudaStream_t st)
{
    TcDenseRun g = {};
    g.x = p.x;
    g.x_stride = p.x_stride;
    g.suh = reinterpret_cast<const __half*>(p.gate_up.suh);
    g.run_input = true;
    g.xt = reinterpret_cast<uint8_t*>(scratch + L.img1);
    g.trellis = p.gate_up.trellis;
    g.svh = reinterpret_cast<const __half*>(p.gate_up.svh);
    g.m = p.m;
    g.k = p.hidden;
    g.n = 2 * p.inter;
    g.K = p.K_gate_up;
    g.cb = p.cb_gate_up;
    g.img = reinterpret_cast<uint8_t*>(scratch + L.img2);
    g.suh2 = reinterpret_cast<const __half*>(p.down.suh);
    g.swiglu_limit = p.swiglu_limit;
    g.slots = reinterpret_cast<float*>(state);
    int rc = tc_dense_run(g, st);
    if (rc != kOk) return rc;

    TcDenseRun d = {};
    d.run_input = false;  // the image was written by the gate|up epilogue
    d.xt = reinterpret_cast<uint8_t*>(scratch + L.img2);
    d.trellis = p.down.trellis;
    d.svh = reinterpret_cast<const __half*>(p.down.svh);
    d.m = p.m;
    d.k = p.inter;
    d.n = p.hidden;
    d.K = p.K_down;
    d.cb = p.cb_down;
    d.out = p.out;
    d.out_stride = p.out_stride;
    d.out_dtype = p.out_dtype;
    d.slots = reinterpret_cast<float*>(state);
    return tc_dense_run(d, st);
}

}  // namespace exl3b200

using namespace exl3b200;

extern "C" int exl3b200_mlp_workspace(int m, int hidden, int inter, int K_gate_up, int cb_gate_up,
                                      size_t* state_bytes, size_t* scratch_bytes)
{
    if (!state_bytes || !scratch_bytes) return kErrNullPointer;
    if (m < 1 || hidden <= 0 || inter <= 0 || hidden % 128 || inter % 128) return kErrBadShape;
    if (K_gate_up < 2 || K_gate_up > 4) return kErrBadBits;
    if (cb_gate_up < 0 || cb_gate_up > 2) return kErrBadCodebook;
    const MlpLayout L = mlp_layout(m, hidden, inter, K_gate_up, cb_gate_up);
    *state_bytes = L.state;
    *scratch_bytes = L.scratch;
    return kOk;
}

extern "C" int exl3b200_mlp(const exl3b200_mlp_args* p, void* state, size_t state_bytes, void* scratch,
                            size_t scratch_bytes, void* stream)
{
    if (!p || !state || !scratch || !p->x || !p->out) return kErrNullPointer;
    const exl3b200_linear& gu = p->gate_up;
    const exl3b200_linear& dn = p->down;
    if (!gu.trellis || !gu.suh || !gu.svh || !dn.trellis || !dn.suh || !dn.svh) return kErrNullPointer;
    if (p->m < 1 || p->hidden <= 0 || p->inter <= 0 || p->hidden % 128 || p->inter % 128) return kErrBadShape;
    if (gu.k != p->hidden || gu.n != 2 * p->inter || dn.k != p->inter || dn.n != p->hidden) return kErrBadShape;
    if (p->x_stride < p->hidden || p->out_stride < p->hidden) return kErrBadShape;
    if (p->K_gate_up < 2 || p->K_gate_up > 4 || p->K_down < 2 || p->K_down > 4) return kErrBadBits;
    if (p->cb_gate_up < 0 || p->cb_gate_up > 2 || p->cb_down < 0 || p->cb_down > 2) return kErrBadCodebook;
    if (p->out_dtype < 0 || p->out_dtype > 2) return kErrBadArgument;
    if (((uintptr_t) p->x & 3) || (p->x_stride & 1) || ((uintptr_t) p->out & 3)) return kErrUnaligned;
    if (((uintptr_t) state & 255) || ((uintptr_t) scratch & 255)) return kErrUnaligned;
    const MlpLayout L = mlp_layout(p->m, p->hidden, p->inter, p->K_gate_up, p->cb_gate_up);
    if (L.tc) {
        const uintptr_t al = (uintptr_t) gu.trellis | (uintptr_t) gu.svh | (uintptr_t) dn.trellis |
                             (uintptr_t) dn.svh | (uintptr_t) dn.suh;
        if (al & 15) return kErrUnaligned;
    } else if (((uintptr_t) gu.trellis | (uintptr_t) dn.trellis) & 3) {
        return kErrUnaligned;
    }
    if (state_bytes < L.state || scratch_bytes < L.scratch) return kErrWorkspace;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    char* sp = reinterpret_cast<char*>(state);
    char* sc = reinterpret_cast<char*>(scratch);
    return L.tc ? mlp_tc(L, *p, sp, sc, st) : mlp_small(L, *p, sp, sc, st);
}
