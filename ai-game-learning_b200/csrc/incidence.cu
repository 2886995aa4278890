// The elementwise part of the incidence residual
// (pbg/games/poker/model/incidence.py:57-84) after its two fp32 card
// contractions: for every decision b, private row r and feature c, over the
// P seats p
//     same_p  = source_p * identical_scale[b, r]
//     oe_p    = sum_q same_q - same_p                        (other_equal)
//     oc_p    = (sum_q overlap_q - overlap_p) - 2 oe_p       (other_card)
//     own_p   = overlap_p - 2 same_p                         (own_card)
// with the seat sums in seat order, as the reference's .sum(1) adds them.
// One pass writes every consumer's copy: oe and own as bf16 into the
// identical / own columns of the incidence map's staged operand, oc as fp32
// (the pre-activation residual of that map's epilogue), and oc^2, oc * oe as
// bf16 into the FamilyFFN operand rows of the token sequence.  A thread owns
// four consecutive features of one (b, r) for all seats (float4 loads).
#include <cuda_bf16.h>

#include "pbg_common.cuh"

namespace pbg {

constexpr int IC_MAXP = 9;  // PokerModelConfig.max_players (preflop.py:80)

__device__ __forceinline__ void ic_store4(__nv_bfloat16* p, float a, float b, float c, float d) {
    __nv_bfloat162 lo = __floats2bfloat162_rn(a, b), hi = __floats2bfloat162_rn(c, d);
    uint2 w;
    w.x = *reinterpret_cast<uint32_t*>(&lo);
    w.y = *reinterpret_cast<uint32_t*>(&hi);
    *reinterpret_cast<uint2*>(p) = w;
}

__global__ void incidence_combine_kernel(int64_t batch, int players, int64_t rows, int d,
                                         const float* __restrict__ source, const float* __restrict__ overlap,
                                         const float* __restrict__ identical_scale, __nv_bfloat16* __restrict__ inc,
                                         int64_t ld_inc, int col_equal, int col_own, float* __restrict__ other_card,
                                         __nv_bfloat16* __restrict__ ffn, int64_t ffn_batch_stride, int64_t ld_ffn,
                                         int col_square, int col_product) {
    const int quads = d >> 2;
    const int64_t item = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (item >= batch * rows * quads) return;
    const int q = (int)(item % quads);
    const int64_t br = item / quads;
    const int64_t b = br / rows, r = br - b * rows;
    const float scale = identical_scale[b * rows + r];
    // pass 1: the seat sums (seat order); pass 2 re-reads each seat's four features (L1-resident) and
    // writes every output, so the thread holds no per-seat arrays
    float4 total_same = make_float4(0.f, 0.f, 0.f, 0.f), total_card = total_same;
    for (int p = 0; p < players; ++p) {
        const int64_t at = ((b * players + p) * rows + r) * d + 4 * q;
        const float4 s = __ldg(reinterpret_cast<const float4*>(source + at));
        const float4 o = __ldg(reinterpret_cast<const float4*>(overlap + at));
        total_same.x += s.x * scale;
        total_same.y += s.y * scale;
        total_same.z += s.z * scale;
        total_same.w += s.w * scale;
        total_card.x += o.x;
        total_card.y += o.y;
        total_card.z += o.z;
        total_card.w += o.w;
    }
    for (int p = 0; p < players; ++p) {
        const int64_t row = (b * players + p) * rows + r;
        const float4 s = __ldg(reinterpret_cast<const float4*>(source + row * d + 4 * q));
        const float4 o = __ldg(reinterpret_cast<const float4*>(overlap + row * d + 4 * q));
        const float4 sm = make_float4(s.x * scale, s.y * scale, s.z * scale, s.w * scale);
        const float4 oe = make_float4(total_same.x - sm.x, total_same.y - sm.y, total_same.z - sm.z,
                                      total_same.w - sm.w);
        const float4 oc = make_float4((total_card.x - o.x) - 2.0f * oe.x, (total_card.y - o.y) - 2.0f * oe.y,
                                      (total_card.z - o.z) - 2.0f * oe.z, (total_card.w - o.w) - 2.0f * oe.w);
        *reinterpret_cast<float4*>(other_card + row * d + 4 * q) = oc;
        __nv_bfloat16* ir = inc + row * ld_inc + 4 * q;
        ic_store4(ir + col_equal, oe.x, oe.y, oe.z, oe.w);
        ic_store4(ir + col_own, o.x - 2.0f * sm.x, o.y - 2.0f * sm.y, o.z - 2.0f * sm.z, o.w - 2.0f * sm.w);
        if (ffn) {
            __nv_bfloat16* fr = ffn + b * ffn_batch_stride + ((int64_t)p * rows + r) * ld_ffn + 4 * q;
            ic_store4(fr + col_square, oc.x * oc.x, oc.y * oc.y, oc.z * oc.z, oc.w * oc.w);
            ic_store4(fr + col_product, oc.x * oe.x, oc.y * oe.y, oc.z * oe.z, oc.w * oe.w);
        }
    }
}

// Backward of incidence_combine_kernel for the same (b, r, 4 features) items: with the output
// gradients g_oe, g_own (bf16 pairs [oe | own] per row), g_oc (fp32) and g_square, g_product (bf16
// [oc^2 | oc oe] per row), each seat's total gradients G_oc = g_oc + 2 oc g_square + oe g_product and
// G_oe = g_oe + oc g_product - 2 G_oc; then d_overlap = (sum G_oc - G_oc) + g_own and
// d_source = ((sum G_oe - G_oe) - 2 g_own) * scale.  Absent gradients (null) are zero.
__device__ __forceinline__ float4 ic_load4(const __nv_bfloat16* p) {
    const uint2 raw = *reinterpret_cast<const uint2*>(p);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
    const float2 a = __bfloat1622float2(h[0]), b = __bfloat1622float2(h[1]);
    return make_float4(a.x, a.y, b.x, b.y);
}

struct IcGrads {
    float4 g_oc, g_oe;
};

__device__ __forceinline__ IcGrads ic_seat_grads(const float4& s, const float4& o, float scale, const float4& ts,
                                                 const float4& tc, const __nv_bfloat16* pair, const float* goc,
                                                 const __nv_bfloat16* sq, int64_t row, int d, int q, float4& g_own) {
    const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
    const float4 ge = pair ? ic_load4(pair + row * 2 * d + 4 * q) : zero;
    g_own = pair ? ic_load4(pair + row * 2 * d + d + 4 * q) : zero;
    const float4 gc = goc ? *reinterpret_cast<const float4*>(goc + row * d + 4 * q) : zero;
    const float4 gs = sq ? ic_load4(sq + row * 2 * d + 4 * q) : zero;
    const float4 gp = sq ? ic_load4(sq + row * 2 * d + d + 4 * q) : zero;
    IcGrads g;
    float* oc_out = &g.g_oc.x;
    float* oe_out = &g.g_oe.x;
    const float* sv = &s.x;
    const float* ov = &o.x;
    const float* tsv = &ts.x;
    const float* tcv = &tc.x;
    const float* gev = &ge.x;
    const float* gcv = &gc.x;
    const float* gsv = &gs.x;
    const float* gpv = &gp.x;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const float oe = tsv[k] - sv[k] * scale;
        const float oc = (tcv[k] - ov[k]) - 2.0f * oe;
        const float goc_total = gcv[k] + 2.0f * oc * gsv[k] + oe * gpv[k];
        oc_out[k] = goc_total;
        oe_out[k] = gev[k] + oc * gpv[k] - 2.0f * goc_total;
    }
    return g;
}

__global__ void incidence_combine_backward_kernel(int64_t batch, int players, int64_t rows, int d,
                                                  const float* __restrict__ source, const float* __restrict__ overlap,
                                                  const float* __restrict__ identical_scale,
                                                  const __nv_bfloat16* __restrict__ g_pair,
                                                  const float* __restrict__ g_other_card,
                                                  const __nv_bfloat16* __restrict__ g_ffn, float* __restrict__ d_source,
                                                  float* __restrict__ d_overlap) {
    const int quads = d >> 2;
    const int64_t item = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (item >= batch * rows * quads) return;
    const int q = (int)(item % quads);
    const int64_t br = item / quads;
    const int64_t b = br / rows, r = br - b * rows;
    const float scale = identical_scale[b * rows + r];
    float4 ts = make_float4(0.f, 0.f, 0.f, 0.f), tc = ts;
    for (int p = 0; p < players; ++p) {
        const int64_t at = ((b * players + p) * rows + r) * d + 4 * q;
        const float4 s = __ldg(reinterpret_cast<const float4*>(source + at));
        const float4 o = __ldg(reinterpret_cast<const float4*>(overlap + at));
        ts.x += s.x * scale;
        ts.y += s.y * scale;
        ts.z += s.z * scale;
        ts.w += s.w * scale;
        tc.x += o.x;
        tc.y += o.y;
        tc.z += o.z;
        tc.w += o.w;
    }
    float4 sum_oc = make_float4(0.f, 0.f, 0.f, 0.f), sum_oe = sum_oc;
    for (int p = 0; p < players; ++p) {
        const int64_t row = (b * players + p) * rows + r;
        const float4 s = __ldg(reinterpret_cast<const float4*>(source + row * d + 4 * q));
        const float4 o = __ldg(reinterpret_cast<const float4*>(overlap + row * d + 4 * q));
        float4 g_own;
        const IcGrads g = ic_seat_grads(s, o, scale, ts, tc, g_pair, g_other_card, g_ffn, row, d, q, g_own);
        sum_oc.x += g.g_oc.x;
        sum_oc.y += g.g_oc.y;
        sum_oc.z += g.g_oc.z;
        sum_oc.w += g.g_oc.w;
        sum_oe.x += g.g_oe.x;
        sum_oe.y += g.g_oe.y;
        sum_oe.z += g.g_oe.z;
        sum_oe.w += g.g_oe.w;
    }
    for (int p = 0; p < players; ++p) {
        const int64_t row = (b * players + p) * rows + r;
        const float4 s = __ldg(reinterpret_cast<const float4*>(source + row * d + 4 * q));
        const float4 o = __ldg(reinterpret_cast<const float4*>(overlap + row * d + 4 * q));
        float4 g_own;
        const IcGrads g = ic_seat_grads(s, o, scale, ts, tc, g_pair, g_other_card, g_ffn, row, d, q, g_own);
        *reinterpret_cast<float4*>(d_overlap + row * d + 4 * q) =
            make_float4(sum_oc.x - g.g_oc.x + g_own.x, sum_oc.y - g.g_oc.y + g_own.y, sum_oc.z - g.g_oc.z + g_own.z,
                        sum_oc.w - g.g_oc.w + g_own.w);
        *reinterpret_cast<float4*>(d_source + row * d + 4 * q) =
            make_float4(((sum_oe.x - g.g_oe.x) - 2.0f * g_own.x) * scale, ((sum_oe.y - g.g_oe.y) - 2.0f * g_own.y) * scale,
                        ((sum_oe.z - g.g_oe.z) - 2.0f * g_own.z) * scale, ((sum_oe.w - g.g_oe.w) - 2.0f * g_own.w) * scale);
    }
}

}  // namespace pbg

using namespace pbg;

extern "C" int pbg_incidence_combine(int64_t batch, int32_t players, int64_t rows, int32_t d, const float* source,
                                     const float* overlap, const float* identical_scale, void* inc, int64_t ld_inc,
                                     int32_t col_equal, int32_t col_own, float* other_card, void* ffn,
                                     int64_t ffn_batch_stride, int64_t ld_ffn, int32_t col_square,
                                     int32_t col_product, void* stream) {
    PBG_REQUIRE(batch >= 0 && rows >= 0 && players >= 1 && players <= IC_MAXP, "incidence_combine: bad shape");
    PBG_REQUIRE(d >= 4 && d % 4 == 0, "incidence_combine: width must be a multiple of 4");
    PBG_REQUIRE(ld_inc % 4 == 0 && col_equal % 4 == 0 && col_own % 4 == 0 && ld_ffn % 4 == 0 &&
                    col_square % 4 == 0 && col_product % 4 == 0 && ffn_batch_stride % 4 == 0,
                "incidence_combine: strides and column offsets must be multiples of 4 elements");
    const int64_t items = batch * rows * (d / 4);
    if (items == 0) return 0;
    PBG_REQUIRE(source && overlap && identical_scale && inc && other_card, "incidence_combine: null pointer");
    PBG_REQUIRE(((uintptr_t)source % 16) == 0 && ((uintptr_t)overlap % 16) == 0 && ((uintptr_t)other_card % 16) == 0 &&
                    ((uintptr_t)inc % 8) == 0 && ((uintptr_t)ffn % 8) == 0,
                "incidence_combine: misaligned buffer");
    incidence_combine_kernel<<<(unsigned)((items + 255) / 256), 256, 0, as_stream(stream)>>>(
        batch, players, rows, d, source, overlap, identical_scale, static_cast<__nv_bfloat16*>(inc), ld_inc,
        col_equal, col_own, other_card, static_cast<__nv_bfloat16*>(ffn), ffn_batch_stride, ld_ffn, col_square,
        col_product);
    return launch_status("incidence_combine");
}

namespace pbg {

// rows of a contiguous bf16 matrix [rows, d] copied into the row block of every sequence of a wider
// buffer: row i -> dst + (i / group_rows) * group_stride + (i % group_rows) * ld (16-byte vectors)
__global__ void scatter_rows_kernel(int64_t rows, int d, int64_t group_rows, const uint4* __restrict__ src,
                                    __nv_bfloat16* __restrict__ dst, int64_t group_stride, int64_t ld) {
    const int vecs = d >> 3;
    const int64_t item = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (item >= rows * vecs) return;
    const int64_t row = item / vecs;
    const int v = (int)(item - row * vecs);
    const int64_t g = row / group_rows, r = row - g * group_rows;
    *reinterpret_cast<uint4*>(dst + g * group_stride + r * ld + 8 * v) = __ldg(src + item);
}

}  // namespace pbg

extern "C" int pbg_scatter_rows_bf16(int64_t rows, int32_t d, int64_t group_rows, const void* src, void* dst,
                                     int64_t group_stride, int64_t ld, void* stream) {
    PBG_REQUIRE(rows >= 0 && d >= 8 && d % 8 == 0 && group_rows >= 1, "scatter_rows: bad shape");
    PBG_REQUIRE(ld % 8 == 0 && group_stride % 8 == 0 && ld >= d, "scatter_rows: strides must be multiples of 8");
    if (rows == 0) return 0;
    PBG_REQUIRE(src && dst && ((uintptr_t)src % 16) == 0 && ((uintptr_t)dst % 16) == 0,
                "scatter_rows: buffers must be 16-byte aligned");
    const int64_t items = rows * (d / 8);
    scatter_rows_kernel<<<(unsigned)((items + 255) / 256), 256, 0, as_stream(stream)>>>(
        rows, d, group_rows, static_cast<const uint4*>(src), static_cast<__nv_bfloat16*>(dst), group_stride, ld);
    return launch_status("scatter_rows_bf16");
}

extern "C" int pbg_incidence_combine_backward(int64_t batch, int32_t players, int64_t rows, int32_t d,
                                              const float* source, const float* overlap, const float* identical_scale,
                                              const void* g_pair, const float* g_other_card, const void* g_ffn,
                                              float* d_source, float* d_overlap, void* stream) {
    PBG_REQUIRE(batch >= 0 && rows >= 0 && players >= 1 && players <= IC_MAXP, "incidence_combine_backward: bad shape");
    PBG_REQUIRE(d >= 4 && d % 4 == 0, "incidence_combine_backward: width must be a multiple of 4");
    const int64_t items = batch * rows * (d / 4);
    if (items == 0) return 0;
    PBG_REQUIRE(source && overlap && identical_scale && d_source && d_overlap, "incidence_combine_backward: null pointer");
    PBG_REQUIRE(((uintptr_t)source | (uintptr_t)overlap | (uintptr_t)d_source | (uintptr_t)d_overlap |
                 (uintptr_t)g_other_card) % 16 == 0 && ((uintptr_t)g_pair | (uintptr_t)g_ffn) % 8 == 0,
                "incidence_combine_backward: misaligned buffer");
    incidence_combine_backward_kernel<<<(unsigned)((items + 255) / 256), 256, 0, as_stream(stream)>>>(
        batch, players, rows, d, source, overlap, identical_scale, static_cast<const __nv_bfloat16*>(g_pair),
        g_other_card, static_cast<const __nv_bfloat16*>(g_ffn), d_source, d_overlap);
    return launch_status("incidence_combine_backward");
}
