// Tile-based front-to-back alpha compositing of projected splats, forward and
// backward.
//
// Reference behaviour: gsplat/cuda/csrc/RasterizeToPixels3DGSFwd.cu:40-213 and
// RasterizeToPixels3DGSBwd.cu:38-301 (per-pixel rules: sigma = 0.5 (a dx^2 +
// c dy^2) + b dx dy, alpha = min(0.99, o exp(-sigma)), skip when sigma < 0 or
// alpha < 1/255, stop before the splat that would take T to <= 1e-4, last_ids =
// index of the last contributing splat; backward walks the same list back to
// front recovering T by division).
//
// Design for sm_100a:
//  * One CTA per (image, tile). Splats of the tile's range are staged in shared
//    memory in batches of 256 as 32-byte records plus their colours.
//  * While staging, each splat gets a conservative pixel-space box of the region
//    where its alpha can reach 1/255. Every warp then compacts the batch into its
//    own list of splats whose box meets the warp's pixel rectangle (ballot +
//    popc), so warps never evaluate splats that cannot touch their pixels.
//    The box is inflated by 1% plus half a pixel; outside it alpha is below the
//    threshold by more than the rounding of the exp evaluation.
//  * Backward threads own 4 pixels each, interleaved for 16x16 tiles (lane l
//    owns pixel l of each 8x4 quarter of its warp's 16x8 rows), so a splat that
//    covers one quarter runs one of the four unrolled per-pixel code blocks.
//    The per-splat gradient is summed over the thread's pixels in registers
//    first. The CDIM + 6 (+ 2 with absgrad) per-splat sums are then reduced over
//    the warp by recursive halving in power-of-two groups (each butterfly step
//    exchanges half of the remaining values), and the finished sums land in
//    different lanes, which issue their atomics in parallel.
//  * The backward recovers T with an approximate reciprocal (__fdividef), as
//    the reference's default fast-math build does.
//  * Channel counts are processed in chunks of at most 32 (kernels are
//    instantiated for 1-8, 16 and 32 channels) with strided colour access, so no
//    padding copies are made.
#include "common.cuh"
#include "gsb_internal.h"

// Compile-time choices of the backward kernel (defaults are the tuned ones).
#ifndef GSB_BWD_MINB
#define GSB_BWD_MINB 14
#endif
#ifndef GSB_BWD_MINB_SMALL
#define GSB_BWD_MINB_SMALL 1
#endif
#ifndef GSB_RAST_FAST_RCP
#define GSB_RAST_FAST_RCP 1
#endif
#ifndef GSB_RAST_INTERLEAVE
#define GSB_RAST_INTERLEAVE 1
#endif
#ifndef GSB_RAST_PAIR
#define GSB_RAST_PAIR 1
#endif



namespace gsb {

#ifndef GSB_RAST_BATCH
#define GSB_RAST_BATCH 128
#endif
constexpr int kBatch = GSB_RAST_BATCH; // splats staged per batch

struct RasterParams {
    uint32_t I, n_isects;
    const float *means2d, *conics, *colors, *opacities, *backgrounds;
    const bool *masks;
    uint32_t W, H, tile_size, tile_w, tile_h;
    const int32_t *offsets, *flatten_ids;
    uint32_t cstride; // floats between consecutive splats' colours (total channels)
    uint32_t coff;    // first channel of this chunk
    // forward outputs
    float *renders; // [I, H, W, cstride]
    float *alphas;  // [I, H, W]
    int32_t *last_ids;
    int32_t *pair_counts; // optional [I, H, W]: splats that contributed to each pixel
    float *final_Ts;      // optional [I, H, W]: final transmittance of each pixel
    bool write_alpha;
    // backward inputs / outputs
    const float *T_final; // optional [I, H, W] final transmittances (else 1 - alphas)
    const float *v_renders, *v_alphas;
    float *v_means2d, *v_conics, *v_colors, *v_opacities, *v_means2d_abs;
    bool first_chunk;
};

// Staged splat: mean, opacity, conic and sig2_max = 2 ln(255 o), twice the
// largest sigma at which alpha = o exp(-sigma) still reaches 1/255.
struct __align__(16) SplatRec {
    float x, y, o, a;
    float b, c, sig2_max, pad1;
};

struct RasterSmem {
    int32_t *ids;
    SplatRec *recs;
    float4 *boxes;
    float *colors;
    uint8_t *lists; // [nwarps][kBatch] 16-bit entries
};

template <int CDIM> __host__ __device__ constexpr size_t raster_smem_bytes(int nwarps) {
    return (size_t)kBatch * sizeof(SplatRec) + (size_t)kBatch * sizeof(float4) +
           (size_t)kBatch * sizeof(int32_t) + (size_t)kBatch * CDIM * sizeof(float) +
           (size_t)nwarps * kBatch * 2;
}

template <int CDIM> __device__ __forceinline__ RasterSmem carve(unsigned char *base) {
    RasterSmem s;
    s.recs = reinterpret_cast<SplatRec *>(base);
    base += kBatch * sizeof(SplatRec);
    s.boxes = reinterpret_cast<float4 *>(base);
    base += kBatch * sizeof(float4);
    s.ids = reinterpret_cast<int32_t *>(base);
    base += kBatch * sizeof(int32_t);
    s.colors = reinterpret_cast<float *>(base);
    base += kBatch * CDIM * sizeof(float);
    s.lists = reinterpret_cast<uint8_t *>(base);
    return s;
}

// Stage splat `g` into slot i: record, colours and the culling box
// (x_min, x_max, y_min, y_max) in pixel-centre coordinates.
template <int CDIM>
__device__ __forceinline__ void stage_splat(const RasterParams &p, const RasterSmem &s, int i,
                                            int32_t g) {
    s.ids[i] = g;
    const float x = p.means2d[(size_t)g * 2], y = p.means2d[(size_t)g * 2 + 1];
    const float a = p.conics[(size_t)g * 3], b = p.conics[(size_t)g * 3 + 1],
                c = p.conics[(size_t)g * 3 + 2];
    const float o = p.opacities[g];
    SplatRec r;
    r.x = x;
    r.y = y;
    r.o = o;
    r.a = a;
    r.b = b;
    r.c = c;
    r.sig2_max = o > 0.f ? 2.f * __logf(o * 255.f) : -1.f;
    r.pad1 = 0.f;
    s.recs[i] = r;
    const float *cp = p.colors + (size_t)g * p.cstride + p.coff;
#pragma unroll
    for (int k = 0; k < CDIM; ++k) s.colors[i * CDIM + k] = cp[k];
    float4 box;
    const float det = a * c - b * b;
    const float o255 = o * 255.f;
    if (det > 0.f && a > 0.f && o255 > 1.0001f) {
        const float lvl = 2.f * __logf(o255);
        const float hx = sqrtf(lvl * c / det) * 1.01f + 0.5f;
        const float hy = sqrtf(lvl * a / det) * 1.01f + 0.5f;
        box = make_float4(x - hx, x + hx, y - hy, y + hy);
    } else if (o255 < 0.9999f && det > 0.f && a > 0.f) {
        box = make_float4(1e30f, -1e30f, 1e30f, -1e30f); // never reaches the threshold
    } else {
        box = make_float4(-1e30f, 1e30f, -1e30f, 1e30f); // no culling
    }
    s.boxes[i] = box;
}

// Pixel-space rectangle of the warp's inside pixels (pixel centres); empty when
// the warp has none.
struct WarpRect {
    float x0, x1, y0, y1;
    bool any;
};

__device__ __forceinline__ WarpRect warp_rect(bool has, float px0, float px1, float py0, float py1) {
    float a = has ? px0 : 1e30f, b = has ? px1 : -1e30f, c = has ? py0 : 1e30f, d = has ? py1 : -1e30f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        a = fminf(a, __shfl_xor_sync(0xffffffffu, a, o));
        b = fmaxf(b, __shfl_xor_sync(0xffffffffu, b, o));
        c = fminf(c, __shfl_xor_sync(0xffffffffu, c, o));
        d = fmaxf(d, __shfl_xor_sync(0xffffffffu, d, o));
    }
    WarpRect r;
    r.x0 = a;
    r.x1 = b;
    r.y0 = c;
    r.y1 = d;
    r.any = __any_sync(0xffffffffu, has);
    return r;
}

__device__ __forceinline__ bool box_hits(const float4 &bx, const WarpRect &r) {
    return !(bx.y < r.x0 || bx.x > r.x1 || bx.w < r.y0 || bx.z > r.y1);
}

// exp(-x / 2) for the pair evaluation: ex2.approx of x * (-log2(e) / 2). The
// product rounds exactly like (x / 2) * log2(e) (halving is exact), so this is
// the hardware exponential of -sigma evaluated the same way as __expf(-sigma).
__device__ __forceinline__ float exp_neg_half(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x * -0.72134752044448170368f));
    return y;
}

// Shared per-pair evaluation: identical in forward and backward so both make the
// same decisions. A pair contributes when sigma >= 0 and alpha = min(0.99,
// o exp(-sigma)) >= 1/255 (reference RasterizeToPixels3DGSFwd.cu:170-176), with
// sigma = 0.5 (a dx^2 + c dy^2) + b dx dy evaluated as half the quadratic form
// d . (conic d): the products g = conic d are the mean gradient's factors too.
// The cheap test 2 sigma > sig2_max = 2 ln(255 o) rejects almost every
// non-contributing pair before the exponential; it is equivalent to alpha <
// 1/255 up to the rounding of the two transcendental evaluations, and the exact
// alpha test is still applied to the pairs that pass it.
// Every operation of the evaluation is rounded explicitly (gx = b dy + (a dx),
// gy = c dy + (b dx), 2 sigma = dy gy + (dx gx), each a fused multiply-add of a
// rounded product), so the scalar form below and the paired form (two pixels
// of one row through sm_100's two-wide FP32 instructions, whose halves round
// like the scalar instructions) give the same bits for a pixel. The forward,
// with two pixels of one row per thread, takes the paired form; the backward
// the scalar one (measured: the paired form there evaluates pixel slots whose
// quarter the splat misses and ran ~3% slower).
struct PairEval {
    float dx, dy, gx, gy, vis, ov, alpha;
    bool keep;
};

__device__ __forceinline__ void finish_pair(const SplatRec &r, float s2, PairEval &e) {
    e.keep = s2 >= 0.f && s2 <= r.sig2_max;
    if (e.keep) {
        e.vis = exp_neg_half(s2);
        e.ov = __fmul_rn(r.o, e.vis);
        e.alpha = fminf(kMaxAlpha, e.ov);
        e.keep = e.alpha >= kAlphaThreshold;
    }
}

__device__ __forceinline__ PairEval eval_pair(const SplatRec &r, float px, float py) {
    PairEval e;
    e.dx = __fsub_rn(r.x, px);
    e.dy = __fsub_rn(r.y, py);
    e.gx = __fmaf_rn(r.b, e.dy, __fmul_rn(r.a, e.dx));
    e.gy = __fmaf_rn(r.c, e.dy, __fmul_rn(r.b, e.dx));
    finish_pair(r, __fmaf_rn(e.dy, e.gy, __fmul_rn(e.dx, e.gx)), e); // 2 sigma
    return e;
}

// Two-wide FP32 operations on a 64-bit register pair (lo, hi).
__device__ __forceinline__ uint64_t f2(float lo, float hi) {
    uint64_t v;
    asm("mov.b64 %0, {%1, %2};" : "=l"(v) : "f"(lo), "f"(hi));
    return v;
}
__device__ __forceinline__ void f2_split(uint64_t v, float &lo, float &hi) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t f2_sub(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}

// A staged splat's fields duplicated into both halves, for the paired form.
struct SplatPair {
    uint64_t x, a, b, c;
};
__device__ __forceinline__ SplatPair splat_pair(const SplatRec &r) {
    SplatPair q;
    q.x = f2(r.x, r.x);
    q.a = f2(r.a, r.a);
    q.b = f2(r.b, r.b);
    q.c = f2(r.c, r.c);
    return q;
}

// eval_pair of the pixels (px.lo, py) and (px.hi, py) of one row.
__device__ __forceinline__ void eval_pair2(const SplatRec &r, const SplatPair &q, uint64_t px, float py,
                                           PairEval &e0, PairEval &e1) {
    const float dy = __fsub_rn(r.y, py);
    const uint64_t DY = f2(dy, dy);
    const uint64_t DX = f2_sub(q.x, px);
    const uint64_t GX = f2_fma(q.b, DY, f2_mul(q.a, DX));
    const uint64_t GY = f2_fma(q.c, DY, f2_mul(q.b, DX));
    const uint64_t S2 = f2_fma(DY, GY, f2_mul(DX, GX));
    float s0, s1;
    f2_split(DX, e0.dx, e1.dx);
    f2_split(GX, e0.gx, e1.gx);
    f2_split(GY, e0.gy, e1.gy);
    f2_split(S2, s0, s1);
    e0.dy = e1.dy = dy;
    finish_pair(r, s0, e0);
    finish_pair(r, s1, e1);
}

// ---------------------------------------------------------------------------
// Forward
// ---------------------------------------------------------------------------
template <int CDIM, int BX, int BY>
__global__ void __launch_bounds__(256) raster_fwd_kernel(RasterParams p) {
    constexpr int PPT = BX * BY;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const RasterSmem s = carve<CDIM>(smem_raw);
    const uint32_t image = blockIdx.y;
    const uint32_t tile = blockIdx.x;
    const uint32_t tx0 = (tile % p.tile_w) * p.tile_size, ty0 = (tile / p.tile_w) * p.tile_size;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;

    float px[PPT], py[PPT], T[PPT], out[PPT][CDIM];
    int32_t cur[PPT], npairs[PPT];
    bool inside[PPT], done[PPT];
    uint32_t pid[PPT];
    bool has = false;
    float rx0 = 1e30f, rx1 = -1e30f, ry0 = 1e30f, ry1 = -1e30f;
#pragma unroll
    for (int k = 0; k < PPT; ++k) {
        // thread owns a BX x BY block of pixels; blocks are laid out row-major
        const uint32_t tpr = p.tile_size / BX;
        const uint32_t ly = (threadIdx.x / tpr) * BY + k / BX, lx = (threadIdx.x % tpr) * BX + k % BX;
        const uint32_t i = ty0 + ly, j = tx0 + lx;
        inside[k] = ly < p.tile_size && i < p.H && j < p.W;
        px[k] = (float)j + 0.5f;
        py[k] = (float)i + 0.5f;
        pid[k] = i * p.W + j;
        T[k] = 1.f;
        cur[k] = 0;
        npairs[k] = 0;
        done[k] = !inside[k];
#pragma unroll
        for (int c = 0; c < CDIM; ++c) out[k][c] = 0.f;
        if (inside[k]) {
            has = true;
            rx0 = fminf(rx0, px[k]);
            rx1 = fmaxf(rx1, px[k]);
            ry0 = fminf(ry0, py[k]);
            ry1 = fmaxf(ry1, py[k]);
        }
    }
    const WarpRect wr = warp_rect(has, rx0, rx1, ry0, ry1);
    const float *bg = p.backgrounds ? p.backgrounds + (size_t)image * p.cstride + p.coff : nullptr;
    constexpr bool kPairFwd = GSB_RAST_PAIR && PPT == 2 && BY == 1;
    const uint64_t px01 = f2(px[0], px[PPT > 1 ? 1 : 0]);

    const size_t tile_flat = (size_t)image * p.tile_w * p.tile_h + tile;
    bool masked = p.masks != nullptr && !p.masks[tile_flat];
    if (!masked) {
        const int32_t start = p.offsets[tile_flat];
        const int32_t end = (image == p.I - 1 && tile == p.tile_w * p.tile_h - 1)
                                ? (int32_t)p.n_isects
                                : p.offsets[tile_flat + 1];
        uint8_t *mylist = s.lists + warp * kBatch * 2;
        for (int32_t bstart = start; bstart < end; bstart += kBatch) {
            bool all_done = true;
#pragma unroll
            for (int k = 0; k < PPT; ++k) all_done &= done[k];
            if (__syncthreads_count(all_done) == (int)blockDim.x) break;
            const int nb = min(kBatch, end - bstart);
            for (int i = threadIdx.x; i < nb; i += blockDim.x)
                stage_splat<CDIM>(p, s, i, p.flatten_ids[bstart + i]);
            __syncthreads();
            // per-warp list of splats that can touch this warp's live pixels
            int cnt = 0;
            const bool warp_live = wr.any && !__all_sync(0xffffffffu, all_done);
            if (warp_live) {
                for (int base = 0; base < nb; base += 32) {
                    const int i = base + lane;
                    const bool hit = i < nb && box_hits(s.boxes[i], wr);
                    const uint32_t bal = __ballot_sync(0xffffffffu, hit);
                    if (hit) mylist[cnt + __popc(bal & ((1u << lane) - 1u))] = (uint8_t)i;
                    cnt += __popc(bal);
                }
            }
            __syncwarp();
            // composite one pair (in list order) into pixel k
            auto apply = [&](int k, const PairEval &e, int i, const float *col) {
                if (!e.keep) return;
                const float next_T = T[k] * (1.f - e.alpha);
                if (next_T <= kTransmittanceThreshold) {
                    done[k] = true;
                    return;
                }
                const float w = e.alpha * T[k];
#pragma unroll
                for (int c = 0; c < CDIM; ++c) out[k][c] += col[c] * w;
                cur[k] = bstart + i;
                ++npairs[k];
                T[k] = next_T;
            };
            for (int li = 0; li < cnt; ++li) {
                bool stop = true;
#pragma unroll
                for (int k = 0; k < PPT; ++k) stop &= done[k];
                if (stop) break;
                const int i = mylist[li];
                const SplatRec r = s.recs[i];
                float col[CDIM];
#pragma unroll
                for (int c = 0; c < CDIM; ++c) col[c] = s.colors[i * CDIM + c];
                if constexpr (kPairFwd) {
                    // the thread's two pixels share a row: one paired evaluation
                    const SplatPair sp = splat_pair(r);
                    PairEval e0, e1;
                    eval_pair2(r, sp, px01, py[0], e0, e1);
                    if (!done[0]) apply(0, e0, i, col);
                    if (!done[1]) apply(1, e1, i, col);
                } else {
#pragma unroll
                    for (int k = 0; k < PPT; ++k) {
                        if (done[k]) continue;
                        apply(k, eval_pair(r, px[k], py[k]), i, col);
                    }
                }
            }

        }
    }
    const size_t img_pix = (size_t)image * p.H * p.W;
#pragma unroll
    for (int k = 0; k < PPT; ++k) {
        if (!inside[k]) continue;
        const size_t pix = img_pix + pid[k];
        float *o = p.renders + pix * p.cstride + p.coff;
        if (masked) {
#pragma unroll
            for (int c = 0; c < CDIM; ++c) o[c] = bg ? bg[c] : 0.f;
            if (p.write_alpha) {
                p.alphas[pix] = 0.f;
                p.last_ids[pix] = 0;
                if (p.pair_counts) p.pair_counts[pix] = 0;
                if (p.final_Ts) p.final_Ts[pix] = 1.f;
            }
            continue;
        }
#pragma unroll
        for (int c = 0; c < CDIM; ++c) o[c] = bg ? out[k][c] + T[k] * bg[c] : out[k][c];
        if (p.write_alpha) {
            p.alphas[pix] = 1.f - T[k];
            p.last_ids[pix] = cur[k];
            if (p.pair_counts) p.pair_counts[pix] = npairs[k];
            if (p.final_Ts) p.final_Ts[pix] = T[k];
        }
    }
}

// ---------------------------------------------------------------------------
// Backward
// ---------------------------------------------------------------------------

// Warp reduction of V values (V a power of two <= 32) by recursive halving: at
// each butterfly step a lane keeps one half of its values and sends the other
// half, so V values cost V - 1 + (5 - log2 V) shuffles instead of 5 V. On return
// the lane holds the complete sum of value `idx`; `writer` marks one lane per
// value. Used for the per-splat gradient sums of the backward pass.
template <int V> struct Log2 { static constexpr int value = 1 + Log2<V / 2>::value; };
template <> struct Log2<1> { static constexpr int value = 0; };

template <int V>
__device__ __forceinline__ float halving_reduce(float *v, int lane, int &idx, bool &writer) {
    constexpr int L = Log2<V>::value;
#pragma unroll
    for (int s = 0; s < L; ++s) {
        const int mask = 16 >> s;
        const int half = V >> (s + 1);
        const bool upper = (lane & mask) != 0;
#pragma unroll
        for (int i = 0; i < half; ++i) {
            const float send = upper ? v[i] : v[i + half];
            const float keep = upper ? v[i + half] : v[i];
            v[i] = keep + __shfl_xor_sync(0xffffffffu, send, mask);
        }
    }
    float r = v[0];
#pragma unroll
    for (int mask = 16 >> L; mask > 0; mask >>= 1) r += __shfl_xor_sync(0xffffffffu, r, mask);
    idx = (lane >> (5 - L)) & (V - 1);
    writer = (lane & ((1 << (5 - L)) - 1)) == 0;
    return r;
}


// Per-splat gradient slots: [0, CDIM) colour, then conic a, b, c, mean x, y,
// opacity, |mean x|, |mean y|. The backward accumulates the conic and mean slots
// without their constant factors (sum of w dx dx, w dx dy, w dy dy, w gx, w gy
// with w = o vis v_alpha = -v_sigma); `scale` restores them on the way out.
template <int CDIM>
__device__ __forceinline__ float *grad_slot(const RasterParams &p, int j, int32_t g, float &scale) {
    scale = 1.f;
    if (j < CDIM) return p.v_colors + (size_t)g * p.cstride + p.coff + j;
    j -= CDIM;
    if (j < 3) {
        scale = j == 1 ? -1.f : -0.5f;
        return p.v_conics + (size_t)g * 3 + j;
    }
    if (j < 5) {
        scale = -1.f;
        return p.v_means2d + (size_t)g * 2 + (j - 3);
    }
    if (j == 5) return p.v_opacities + g;
    return p.v_means2d_abs ? p.v_means2d_abs + (size_t)g * 2 + (j - 6) : nullptr;
}

// Reduces slots [FIRST, FIRST + COUNT) over the warp and adds them to the
// splat's gradients: the largest power-of-two group by recursive halving, the
// rest recursively (8 + 1 slots cost fewer instructions than 16 padded ones).
template <int CDIM, int FIRST, int COUNT>
__device__ __forceinline__ void flush_range(const RasterParams &p, const float *acc, int lane, int32_t g) {
    if constexpr (COUNT > 0) {
        constexpr int V = COUNT >= 32 ? 32 : (COUNT >= 16 ? 16 : (COUNT >= 8 ? 8 : (COUNT >= 4 ? 4 : (COUNT >= 2 ? 2 : 1))));
        float v[V];
#pragma unroll
        for (int i = 0; i < V; ++i) v[i] = acc[FIRST + i];
        int idx;
        bool writer;
        const float r = halving_reduce<V>(v, lane, idx, writer);
        if (writer) {
            float scale;
            float *dst = grad_slot<CDIM>(p, FIRST + idx, g, scale);
            if (dst) atomicAdd(dst, r * scale);
        }
        flush_range<CDIM, FIRST + V, COUNT - V>(p, acc, lane, g);
    }
}

template <int CDIM, int NV>
__device__ __forceinline__ void flush_splat_grads(const RasterParams &p, const float *acc, int lane,
                                                  int32_t g) {
    flush_range<CDIM, 0, NV>(p, acc, lane, g);
}

// ABS: accumulate |v_mean2d| per pair (absgrad). IL: interleaved pixel layout
// for 16x16 tiles with 4 pixels per thread: warp w covers rows 8w .. 8w + 7 as
// four 8x4 quarters and lane l owns pixel (l % 8, l / 8) of every quarter, so a
// splat whose culling box misses a quarter skips that pixel slot in every lane
// (a warp-uniform branch: the quarter mask is computed once per splat and warp).
//
// Per pixel the backward keeps T (recovered back to front), S = buf . v_colour
// - tv (buf: the colour behind the current splat, only ever needed dotted with
// the upstream colour gradient; tv = T_final (v_alpha - bg . v_colour), folded in
// once), the upstream colour gradient and the last contributor. With cv =
// colour . v_colour the reference's v_alpha = sum_c (colour_c T - buf_c ra) v_c
// + ra tv becomes T cv - ra S, and S grows by alpha T cv.
template <int CDIM, int BX, int BY, bool ABS, bool IL>
__global__ void __launch_bounds__(256 / (BX * BY), (BX * BY >= 4 ? (CDIM <= 3 ? GSB_BWD_MINB : 8) : GSB_BWD_MINB_SMALL))
    raster_bwd_kernel(RasterParams p) {
    constexpr int PPT = BX * BY;
    static_assert(!IL || PPT == 4, "interleaved layout: 4 pixels per thread");
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const RasterSmem s = carve<CDIM>(smem_raw);
    const uint32_t image = blockIdx.y;
    const uint32_t tile = blockIdx.x;
    const size_t tile_flat = (size_t)image * p.tile_w * p.tile_h + tile;
    if (p.masks != nullptr && !p.masks[tile_flat]) return;
    const uint32_t tx0 = (tile % p.tile_w) * p.tile_size, ty0 = (tile / p.tile_w) * p.tile_size;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const size_t img_pix = (size_t)image * p.H * p.W;
    const float *bg = p.backgrounds ? p.backgrounds + (size_t)image * p.cstride + p.coff : nullptr;

    float px[PPT], py[PPT], T[PPT], S[PPT], vc[PPT][CDIM], tv[PPT];
    int32_t bin_final[PPT];
    bool has = false;
    int32_t my_max = -1;
    float rx0 = 1e30f, rx1 = -1e30f, ry0 = 1e30f, ry1 = -1e30f;
#pragma unroll
    for (int k = 0; k < PPT; ++k) {
        uint32_t ly, lx;
        if (IL) {
            ly = warp * 8 + (k >> 1) * 4 + (lane >> 3);
            lx = (k & 1) * 8 + (lane & 7);
        } else {
            // thread owns a BX x BY block of pixels; blocks are laid out row-major
            const uint32_t tpr = p.tile_size / BX;
            ly = (threadIdx.x / tpr) * BY + k / BX;
            lx = (threadIdx.x % tpr) * BX + k % BX;
        }
        const uint32_t i = ty0 + ly, j = tx0 + lx;
        const bool inside = ly < p.tile_size && i < p.H && j < p.W;
        px[k] = (float)j + 0.5f;
        py[k] = (float)i + 0.5f;
        const size_t pix = img_pix + (inside ? i * p.W + j : 0);
        // The final transmittance saved by the forward when given; 1 - alpha
        // otherwise (the reference's form, which loses the low bits of T when
        // the pixel is nearly opaque: alpha = 0.9999 carries T to ~3e-4).
        const float Tf = inside ? (p.T_final ? p.T_final[pix] : 1.f - p.alphas[pix]) : 0.f;
        T[k] = Tf;
        bin_final[k] = inside ? p.last_ids[pix] : -1;
        float dotbg = 0.f;
#pragma unroll
        for (int c = 0; c < CDIM; ++c) {
            vc[k][c] = inside ? p.v_renders[pix * p.cstride + p.coff + c] : 0.f;
            if (bg) dotbg += bg[c] * vc[k][c];
        }
        const float va = (inside && p.first_chunk) ? p.v_alphas[pix] : 0.f;
        tv[k] = Tf * (va - dotbg);
        S[k] = -tv[k]; // S - tv, accumulated directly
        if (inside) {
            has = true;
            my_max = max(my_max, bin_final[k]);
            rx0 = fminf(rx0, px[k]);
            rx1 = fmaxf(rx1, px[k]);
            ry0 = fminf(ry0, py[k]);
            ry1 = fmaxf(ry1, py[k]);
        }
    }
    const WarpRect wr = warp_rect(has, rx0, rx1, ry0, ry1);
    int32_t warp_max = my_max;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) warp_max = max(warp_max, __shfl_xor_sync(0xffffffffu, warp_max, o));
    // pixel-centre rectangles of the warp's four quarters (interleaved layout)
    const float qx0 = (float)tx0 + 0.5f, qy0 = (float)(ty0 + warp * 8) + 0.5f;

    const int32_t start = p.offsets[tile_flat];
    const int32_t end = (image == p.I - 1 && tile == p.tile_w * p.tile_h - 1) ? (int32_t)p.n_isects
                                                                              : p.offsets[tile_flat + 1];
    // Splats behind every pixel's last contributor in the whole block are skipped.
    __shared__ int32_t block_max_s;
    if (threadIdx.x == 0) block_max_s = -1;
    __syncthreads();
    if (lane == 0 && wr.any) atomicMax(&block_max_s, warp_max);
    __syncthreads();
    const int32_t block_max = block_max_s;
    const int32_t last = min(end - 1, block_max);
    uint8_t *mylist = s.lists + warp * kBatch * 2;
    for (int32_t bend = last; bend >= start; bend -= kBatch) {
        const int nb = min(kBatch, bend + 1 - start);
        __syncthreads();
        for (int i = threadIdx.x; i < nb; i += blockDim.x)
            stage_splat<CDIM>(p, s, i, p.flatten_ids[bend - i]);
        __syncthreads();
        // per-warp list of the splats whose box meets the warp's pixels, with
        // the quarters they meet (bits 8..11 of each 16-bit entry)
        int cnt = 0;
        uint16_t *mylist16 = reinterpret_cast<uint16_t *>(mylist);
        if (wr.any) {
            for (int base = 0; base < nb; base += 32) {
                const int i = base + lane;
                uint32_t q = 0;
                if (i < nb && (bend - i) <= warp_max) {
                    const float4 bx = s.boxes[i];
                    if (box_hits(bx, wr)) {
                        if (IL) {
#pragma unroll
                            for (int k = 0; k < 4; ++k) {
                                const float x0 = qx0 + (k & 1) * 8, y0 = qy0 + (k >> 1) * 4;
                                if (!(bx.y < x0 || bx.x > x0 + 7.f || bx.w < y0 || bx.z > y0 + 3.f)) q |= 1u << k;
                            }
                        } else {
                            q = 0xfu;
                        }
                    }
                }
                const bool hit = q != 0;
                const uint32_t bal = __ballot_sync(0xffffffffu, hit);
                if (hit) mylist16[cnt + __popc(bal & ((1u << lane) - 1u))] = (uint16_t)(i | (q << 8));
                cnt += __popc(bal);
            }
        }
        __syncwarp();
        for (int li = 0; li < cnt; ++li) {
            const uint32_t ent = mylist16[li];
            const int i = ent & 0xff;
            const uint32_t qmask = ent >> 8;
            const int32_t gidx = bend - i;
            constexpr int NV = CDIM + (ABS ? 8 : 6);
            float acc[NV];
#pragma unroll
            for (int j = 0; j < NV; ++j) acc[j] = 0.f;
            bool any = false;
            const SplatRec r = s.recs[i];
            float col[CDIM];
#pragma unroll
            for (int c = 0; c < CDIM; ++c) col[c] = s.colors[i * CDIM + c];
            // the kept pair's contribution to the splat's sums and to pixel k's state
            auto add_pair = [&](const int k, const PairEval &e) {
                any = true;
#if GSB_RAST_FAST_RCP
                // approximate reciprocal, as the reference's default fast-math build
                const float ra = __fdividef(1.f, fmaxf(kMinOneMinusAlpha, 1.f - e.alpha));
#else
                const float ra = 1.f / fmaxf(kMinOneMinusAlpha, 1.f - e.alpha);
#endif
                T[k] *= ra;
                const float fac = e.alpha * T[k];
                float cv = 0.f;
#pragma unroll
                for (int c = 0; c < CDIM; ++c) {
                    acc[c] += fac * vc[k][c];
                    cv += col[c] * vc[k][c];
                }
                const float v_alpha = T[k] * cv - ra * S[k];
                {
                    // no gradient through the opacity and the footprint where the
                    // alpha clamp is active (a select instead of a branch)
                    const bool g = e.ov <= kMaxAlpha;
                    const float w = g ? e.ov * v_alpha : 0.f; // -v_sigma
                    const float wx = w * e.dx, wy = w * e.dy;
                    acc[CDIM + 0] += wx * e.dx;
                    acc[CDIM + 1] += wx * e.dy;
                    acc[CDIM + 2] += wy * e.dy;
                    const float gx = w * e.gx, gy = w * e.gy;
                    acc[CDIM + 3] += gx;
                    acc[CDIM + 4] += gy;
                    acc[CDIM + 5] += (g ? e.vis : 0.f) * v_alpha;
                    if constexpr (ABS) {
                        acc[CDIM + 6] += fabsf(gx);
                        acc[CDIM + 7] += fabsf(gy);
                    }
                }
                S[k] += fac * cv;
            };
#pragma unroll
            for (int k = 0; k < PPT; ++k) {
                if (IL && !(qmask & (1u << k))) continue;
                if (gidx > bin_final[k]) continue;
                const PairEval e = eval_pair(r, px[k], py[k]);
                if (!e.keep) continue;
                add_pair(k, e);
            }
            if (!__any_sync(0xffffffffu, any)) continue;
            flush_splat_grads<CDIM, NV>(p, acc, lane, s.ids[i]);
        }
    }
}

// ---------------------------------------------------------------------------
// Host launchers
// ---------------------------------------------------------------------------
static int threads_for(uint32_t tile_size, int ppt) {
    const uint32_t pix = tile_size * tile_size;
    uint32_t t = (pix + ppt - 1) / ppt;
    t = (t + 31) / 32 * 32;
    return (int)t;
}

template <int CDIM, int BX, int BY>
static int launch_variant(bool fwd, const RasterParams &p, cudaStream_t stream) {
    const int nt = threads_for(p.tile_size, BX * BY);
    if (nt > 256) return set_error(kErrUnsupported, "tile_size %u too large", p.tile_size);
    const size_t smem = raster_smem_bytes<CDIM>(nt / 32);
    dim3 grid(p.tile_w * p.tile_h, p.I);
    if (fwd) {
        auto kern = raster_fwd_kernel<CDIM, BX, BY>;
        if (smem > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        kern<<<grid, nt, smem, stream>>>(p);
        return check_launch("raster_fwd_kernel");
    }
    auto run = [&](auto kern) {
        if (smem > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        kern<<<grid, nt, smem, stream>>>(p);
        return check_launch("raster_bwd_kernel");
    };
    constexpr bool kCanInterleave = GSB_RAST_INTERLEAVE && BX * BY == 4;
    const bool il = kCanInterleave && p.tile_size == 16;
    const bool abs = p.v_means2d_abs != nullptr;
    if (il) {
        return abs ? run(raster_bwd_kernel<CDIM, BX, BY, true, kCanInterleave>)
                   : run(raster_bwd_kernel<CDIM, BX, BY, false, kCanInterleave>);
    }
    return abs ? run(raster_bwd_kernel<CDIM, BX, BY, true, false>)
               : run(raster_bwd_kernel<CDIM, BX, BY, false, false>);
}

// Pixel blocks per thread (BX x BY). Backward: enough pixels per thread to
// amortise the warp reduction, few enough that the per-pixel state
// (transmittance, colour buffer, upstream gradient) stays in registers. Both
// need the tile size to be a multiple of the block; other tile sizes use 1x1.
#ifndef GSB_FWD_BX
#define GSB_FWD_BX 2
#define GSB_FWD_BY 1
#endif
#ifndef GSB_BWD_BX
#define GSB_BWD_BX 4
#define GSB_BWD_BY 1
#endif

template <int CDIM>
static int launch_fwd(const RasterParams &p, cudaStream_t stream) {
    constexpr int BX = GSB_FWD_BX, BY = GSB_FWD_BY;
    if (p.tile_size % BX == 0 && p.tile_size % BY == 0 && p.tile_size >= 8)
        return launch_variant<CDIM, BX, BY>(true, p, stream);
    return launch_variant<CDIM, 1, 1>(true, p, stream);
}

template <int CDIM>
static int launch_bwd(const RasterParams &p, cudaStream_t stream) {
    constexpr int BX = CDIM <= 4 ? GSB_BWD_BX : (CDIM <= 8 ? 2 : 1);
    constexpr int BY = CDIM <= 4 ? GSB_BWD_BY : 1;
    static_assert(BX * BY <= 8, "pixels per thread");
    if (p.tile_size % BX == 0 && p.tile_size % BY == 0 && p.tile_size >= 8)
        return launch_variant<CDIM, BX, BY>(false, p, stream);
    return launch_variant<CDIM, 1, 1>(false, p, stream);
}

template <bool FWD> static int dispatch(int cdim, const RasterParams &p, cudaStream_t s) {
#define GSB_CASE(N)                                                                               \
    case N: return FWD ? launch_fwd<N>(p, s) : launch_bwd<N>(p, s);
    switch (cdim) {
        GSB_CASE(1)
        GSB_CASE(2)
        GSB_CASE(3)
        GSB_CASE(4)
        GSB_CASE(5)
        GSB_CASE(6)
        GSB_CASE(7)
        GSB_CASE(8)
        GSB_CASE(16)
        GSB_CASE(32)
    default: return set_error(kErrUnsupported, "Unsupported number of channels: %d", cdim);
    }
#undef GSB_CASE
}

// Splits `channels` into kernel chunks: 32s, then a 16, an 8, and the rest.
static int next_chunk(int remaining) {
    if (remaining >= 32) return 32;
    if (remaining >= 16) return 16;
    if (remaining >= 8) return 8;
    return remaining;
}

static int check_raster_args(int I, int W, int H, int tile_size, int tile_w, int tile_h, int channels) {
    if (channels <= 0) return set_error(kErrInvalidArgument, "Unsupported number of channels: %d", channels);
    if (tile_size <= 0 || tile_size > 16)
        return set_error(kErrUnsupported, "tile_size %d not supported (1..16)", tile_size);
    if ((long long)tile_w * tile_size < W || (long long)tile_h * tile_size < H)
        return set_error(kErrInvalidArgument, "tile grid %dx%d of size %d does not cover %dx%d", tile_w,
                         tile_h, tile_size, W, H);
    if (I < 0) return set_error(kErrInvalidArgument, "negative image count");
    return kOk;
}

} // namespace gsb

using namespace gsb;

static int rasterize_fwd(int I, int channels, const float *means2d, const float *conics,
                         const float *colors, const float *opacities, const float *backgrounds,
                         const bool *masks, int width, int height, int tile_size, int tile_width,
                         int tile_height, const int32_t *tile_offsets, const int32_t *flatten_ids,
                         long long n_isects, float *renders, float *alphas, int32_t *last_ids,
                         float *final_Ts, int32_t *pair_counts, cudaStream_t stream) {
    if (int e = check_raster_args(I, width, height, tile_size, tile_width, tile_height, channels)) return e;
    if (I == 0 || width == 0 || height == 0) return kOk;
    RasterParams p = {};
    p.I = I;
    p.n_isects = (uint32_t)n_isects;
    p.means2d = means2d;
    p.conics = conics;
    p.colors = colors;
    p.opacities = opacities;
    p.backgrounds = backgrounds;
    p.masks = masks;
    p.W = width;
    p.H = height;
    p.tile_size = tile_size;
    p.tile_w = tile_width;
    p.tile_h = tile_height;
    p.offsets = tile_offsets;
    p.flatten_ids = flatten_ids;
    p.cstride = channels;
    p.renders = renders;
    p.alphas = alphas;
    p.last_ids = last_ids;
    p.pair_counts = pair_counts;
    p.final_Ts = final_Ts;
    int coff = 0;
    while (coff < channels) {
        const int n = next_chunk(channels - coff);
        p.coff = coff;
        p.write_alpha = coff == 0;
        if (int e = dispatch<true>(n, p, stream)) return e;
        coff += n;
    }
    return kOk;
}

extern "C" int gsb_rasterize_fwd(int I, int channels, const float *means2d, const float *conics,
                                 const float *colors, const float *opacities,
                                 const float *backgrounds, const bool *masks, int width, int height,
                                 int tile_size, int tile_width, int tile_height,
                                 const int32_t *tile_offsets, const int32_t *flatten_ids,
                                 long long n_isects, float *renders, float *alphas,
                                 int32_t *last_ids, cudaStream_t stream) {
    return rasterize_fwd(I, channels, means2d, conics, colors, opacities, backgrounds, masks, width,
                         height, tile_size, tile_width, tile_height, tile_offsets, flatten_ids,
                         n_isects, renders, alphas, last_ids, nullptr, nullptr, stream);
}

extern "C" int gsb_rasterize_fwd_counted(int I, int channels, const float *means2d,
                                         const float *conics, const float *colors,
                                         const float *opacities, const float *backgrounds,
                                         const bool *masks, int width, int height, int tile_size,
                                         int tile_width, int tile_height,
                                         const int32_t *tile_offsets, const int32_t *flatten_ids,
                                         long long n_isects, float *renders, float *alphas,
                                         int32_t *last_ids, int32_t *pair_counts,
                                         cudaStream_t stream) {
    return rasterize_fwd(I, channels, means2d, conics, colors, opacities, backgrounds, masks, width,
                         height, tile_size, tile_width, tile_height, tile_offsets, flatten_ids,
                         n_isects, renders, alphas, last_ids, nullptr, pair_counts, stream);
}

extern "C" int gsb_rasterize_fwd_ex(int I, int channels, const float *means2d, const float *conics,
                                    const float *colors, const float *opacities,
                                    const float *backgrounds, const bool *masks, int width,
                                    int height, int tile_size, int tile_width, int tile_height,
                                    const int32_t *tile_offsets, const int32_t *flatten_ids,
                                    long long n_isects, float *renders, float *alphas,
                                    int32_t *last_ids, float *final_Ts, int32_t *pair_counts,
                                    cudaStream_t stream) {
    return rasterize_fwd(I, channels, means2d, conics, colors, opacities, backgrounds, masks, width,
                         height, tile_size, tile_width, tile_height, tile_offsets, flatten_ids,
                         n_isects, renders, alphas, last_ids, final_Ts, pair_counts, stream);
}

static int rasterize_bwd(int I, int channels, const float *means2d, const float *conics,
                         const float *colors, const float *opacities, const float *backgrounds,
                         const bool *masks, int width, int height, int tile_size, int tile_width,
                         int tile_height, const int32_t *tile_offsets, const int32_t *flatten_ids,
                         long long n_isects, const float *render_alphas, const float *final_Ts,
                         const int32_t *last_ids, const float *v_render_colors,
                         const float *v_render_alphas, float *v_means2d_abs, float *v_means2d,
                         float *v_conics, float *v_colors, float *v_opacities, cudaStream_t stream) {
    if (int e = check_raster_args(I, width, height, tile_size, tile_width, tile_height, channels)) return e;
    if (I == 0 || width == 0 || height == 0 || n_isects <= 0) return kOk;
    RasterParams p = {};
    p.I = I;
    p.n_isects = (uint32_t)n_isects;
    p.means2d = means2d;
    p.conics = conics;
    p.colors = colors;
    p.opacities = opacities;
    p.backgrounds = backgrounds;
    p.masks = masks;
    p.W = width;
    p.H = height;
    p.tile_size = tile_size;
    p.tile_w = tile_width;
    p.tile_h = tile_height;
    p.offsets = tile_offsets;
    p.flatten_ids = flatten_ids;
    p.cstride = channels;
    p.alphas = const_cast<float *>(render_alphas);
    p.T_final = final_Ts;
    p.last_ids = const_cast<int32_t *>(last_ids);
    p.v_renders = v_render_colors;
    p.v_alphas = v_render_alphas;
    p.v_means2d = v_means2d;
    p.v_conics = v_conics;
    p.v_colors = v_colors;
    p.v_opacities = v_opacities;
    p.v_means2d_abs = v_means2d_abs;
    int coff = 0;
    while (coff < channels) {
        const int n = next_chunk(channels - coff);
        p.coff = coff;
        p.first_chunk = coff == 0;
        if (int e = dispatch<false>(n, p, stream)) return e;
        coff += n;
    }
    return kOk;
}

extern "C" int gsb_rasterize_bwd(int I, int channels, const float *means2d, const float *conics,
                                 const float *colors, const float *opacities,
                                 const float *backgrounds, const bool *masks, int width, int height,
                                 int tile_size, int tile_width, int tile_height,
                                 const int32_t *tile_offsets, const int32_t *flatten_ids,
                                 long long n_isects, const float *render_alphas,
                                 const int32_t *last_ids, const float *v_render_colors,
                                 const float *v_render_alphas, float *v_means2d_abs,
                                 float *v_means2d, float *v_conics, float *v_colors,
                                 float *v_opacities, cudaStream_t stream) {
    return rasterize_bwd(I, channels, means2d, conics, colors, opacities, backgrounds, masks, width,
                         height, tile_size, tile_width, tile_height, tile_offsets, flatten_ids,
                         n_isects, render_alphas, nullptr, last_ids, v_render_colors,
                         v_render_alphas, v_means2d_abs, v_means2d, v_conics, v_colors, v_opacities,
                         stream);
}

extern "C" int gsb_rasterize_bwd_ex(int I, int channels, const float *means2d, const float *conics,
                                    const float *colors, const float *opacities,
                                    const float *backgrounds, const bool *masks, int width,
                                    int height, int tile_size, int tile_width, int tile_height,
                                    const int32_t *tile_offsets, const int32_t *flatten_ids,
                                    long long n_isects, const float *render_alphas,
                                    const float *final_Ts, const int32_t *last_ids,
                                    const float *v_render_colors, const float *v_render_alphas,
                                    float *v_means2d_abs, float *v_means2d, float *v_conics,
                                    float *v_colors, float *v_opacities, cudaStream_t stream) {
    return rasterize_bwd(I, channels, means2d, conics, colors, opacities, backgrounds, masks, width,
                         height, tile_size, tile_width, tile_height, tile_offsets, flatten_ids,
                         n_isects, render_alphas, final_Ts, last_ids, v_render_colors,
                         v_render_alphas, v_means2d_abs, v_means2d, v_conics, v_colors, v_opacities,
                         stream);
}
