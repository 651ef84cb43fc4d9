// Decision inputs of the ShadowKV agent on the device:
//
//  * skv_reuse_decide     ShadowKVAgent.decide_reuse_per_token (shadowinfer/shadowkv/shadowkv_agent.py:1165-1256):
//                         relative L2 drift of K and V per (token, head), norms over (batch, head_dim),
//                         against the importance-scaled threshold; mask [S,H] plus the per-token
//                         full / partial / none counts, in one pass over the four K/V tensors.
//  * skv_irap_importance  compute_irap_importance (shadowinfer/shadowkv/importance_model.py:37-134), with
//                         the agent's input contract (softmax of logits / row-sum correction,
//                         shadowkv_agent.py:894-965): one pass over the attention weights gives the
//                         received attention (column sums over batch and queries) and each query
//                         row's entropy terms (sum c and sum c*ln c of c = max(w, 1e-10) over batch and
//                         keys); small kernels then form the EMA, the per-head stable rank of the EMA
//                         and the blended importance.
//
// Reductions are deterministic (fixed order) and at least as accurate as the reference's float32
// torch reductions: float64 accumulation of float32 partials of a few terms, or compensated
// float32 sums; the steps the reference does elementwise in float32 (the EMA, the drift ratios)
// are done in float32 with the reference's roundings (no contraction into FMAs).
#include <float.h>
#include <math.h>
#include <stddef.h>

#include "skv_common.cuh"

namespace skv {

// ------------------------------------------------------------------------------ reuse decision
constexpr int kReuseTokens = 2;     // tokens per block (all their heads)

__device__ __forceinline__ double warp_sum_d(double x) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
    return x;
}

// Sums 8 doubles over the warp with a transpose-reduce butterfly (9 double shuffles): lane L
// ends with the full sum of value ((L >> 4) & 1) * 4 + ((L >> 3) & 1) * 2 + ((L >> 2) & 1).
__device__ __forceinline__ double warp_sum8d(const double (&v)[8], int lane) {
    double a[4], b[2];
    const bool h16 = lane & 16, h8 = lane & 8, h4 = lane & 4;
#pragma unroll
    for (int i = 0; i < 4; ++i)
        a[i] = (h16 ? v[i + 4] : v[i]) + __shfl_xor_sync(0xffffffffu, h16 ? v[i] : v[i + 4], 16);
#pragma unroll
    for (int i = 0; i < 2; ++i)
        b[i] = (h8 ? a[i + 2] : a[i]) + __shfl_xor_sync(0xffffffffu, h8 ? a[i] : a[i + 2], 8);
    double c = (h4 ? b[1] : b[0]) + __shfl_xor_sync(0xffffffffu, h4 ? b[0] : b[1], 4);
    c += __shfl_xor_sync(0xffffffffu, c, 2);
    c += __shfl_xor_sync(0xffffffffu, c, 1);
    return c;
}

// This lane's share of one entry's four sums of squares: |k - k_prev|^2, |k|^2, |v - v_prev|^2,
// |v|^2 over (batch, head_dim).  Vector path: float32 partials of four squares (relative error
// < 2^-22), one float64 add per tensor, a quarter of the float32 -> float64 conversions.
__device__ __forceinline__ void entry_sums(const float* __restrict__ kc, const float* __restrict__ vc,
                                           const float* __restrict__ kp, const float* __restrict__ vp, int B, int H,
                                           int S, int D, int t, int h, int lane, bool vec, double* out) {
    double sdk = 0.0, sck = 0.0, sdv = 0.0, scv = 0.0;
    for (int b = 0; b < B; ++b) {
        const int64_t row = (((int64_t)b * H + h) * S + t) * D;
        if (vec) {
            for (int d = lane * 4; d < D; d += 128) {
                const float4 a = __ldg(reinterpret_cast<const float4*>(kc + row + d));
                const float4 a0 = __ldg(reinterpret_cast<const float4*>(kp + row + d));
                const float4 c = __ldg(reinterpret_cast<const float4*>(vc + row + d));
                const float4 c0 = __ldg(reinterpret_cast<const float4*>(vp + row + d));
                const float ka[4] = {a.x, a.y, a.z, a.w}, kb[4] = {a0.x, a0.y, a0.z, a0.w};
                const float va[4] = {c.x, c.y, c.z, c.w}, vb[4] = {c0.x, c0.y, c0.z, c0.w};
                float fdk = 0.f, fck = 0.f, fdv = 0.f, fcv = 0.f;
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const float dk = __fsub_rn(ka[i], kb[i]), dv = __fsub_rn(va[i], vb[i]);
                    fdk = fmaf(dk, dk, fdk);
                    fck = fmaf(ka[i], ka[i], fck);
                    fdv = fmaf(dv, dv, fdv);
                    fcv = fmaf(va[i], va[i], fcv);
                }
                sdk += (double)fdk;
                sck += (double)fck;
                sdv += (double)fdv;
                scv += (double)fcv;
            }
        } else {
            for (int d = lane; d < D; d += 32) {
                const float ka = __ldg(kc + row + d), kb = __ldg(kp + row + d);
                const float va = __ldg(vc + row + d), vb = __ldg(vp + row + d);
                const double dk = (double)__fsub_rn(ka, kb), dv = (double)__fsub_rn(va, vb);
                sdk = fma(dk, dk, sdk);
                sck = fma((double)ka, (double)ka, sck);
                sdv = fma(dv, dv, sdv);
                scv = fma((double)va, (double)va, scv);
            }
        }
    }
    out[0] = sdk;
    out[1] = sck;
    out[2] = sdv;
    out[3] = scv;
}

// Block: kReuseTokens tokens x all H heads; a warp takes two (token, head) entries at a time
// (entries e and e + 8), loads both before reducing, and reduces their eight sums together.
__global__ void __launch_bounds__(256) reuse_decide_kernel(const float* __restrict__ kc, const float* __restrict__ vc,
                                                          const float* __restrict__ kp, const float* __restrict__ vp,
                                                          int B, int H, int S, int D,
                                                          const float* __restrict__ importance, double eff,
                                                          uint8_t* __restrict__ mask, float* __restrict__ drift,
                                                          unsigned long long* __restrict__ counts) {
    extern __shared__ uint8_t s_mask[];             // [kReuseTokens * H]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t0 = blockIdx.x * kReuseTokens;
    const int nt = min(kReuseTokens, S - t0);
    const int ne = nt * H;
    const bool vec = (D & 3) == 0;
    for (int e0 = warp; e0 < ne; e0 += 16) {
        double v[8];
        entry_sums(kc, vc, kp, vp, B, H, S, D, t0 + e0 / H, e0 % H, lane, vec, v);
        const int e1 = e0 + 8;
        if (e1 < ne) {
            entry_sums(kc, vc, kp, vp, B, H, S, D, t0 + e1 / H, e1 % H, lane, vec, v + 4);
        } else {
            v[4] = v[5] = v[6] = v[7] = 0.0;
        }
        // lanes 0-15 hold the entry-e0 sums (value vi in lanes 4vi..4vi+3), lanes 16-31 entry e1
        const double c = warp_sum8d(v, lane);
        const double s1 = __shfl_down_sync(0xffffffffu, c, 4);
        const double s2 = __shfl_down_sync(0xffffffffu, c, 8);
        const double s3 = __shfl_down_sync(0xffffffffu, c, 12);
        const int e = lane == 0 ? e0 : e1;
        if ((lane == 0 || lane == 16) && e < ne) {
            const int t = t0 + e / H, h = e % H;
            const double sdk = c, sck = s1, sdv = s2, scv = s3;
            // float32 norms, then the reference's float32 steps: (|dk| / (|k| + 1e-8) + ...) / 2
            const float nk = __fadd_rn((float)sqrt(sck), 1e-8f), nv = __fadd_rn((float)sqrt(scv), 1e-8f);
            const float dk = __fdiv_rn((float)sqrt(sdk), nk), dv = __fdiv_rn((float)sqrt(sdv), nv);
            const float delta = __fdiv_rn(__fadd_rn(dk, dv), 2.0f);
            // threshold in float64: eff * (1 - 0.3 * clamp(imp, 0, 1)), at least 1e-5 (NaN stays NaN)
            double imp = (double)importance[(int64_t)t * H + h];
            double thr;
            if (imp != imp) {
                thr = imp;
            } else {
                imp = fmin(fmax(imp, 0.0), 1.0);
                thr = __dmul_rn(eff, __dsub_rn(1.0, __dmul_rn(0.3, imp)));
                thr = thr != thr ? thr : fmax(thr, 1e-5);
            }
            const uint8_t m = ((double)delta < thr) ? 1 : 0;
            mask[(int64_t)t * H + h] = m;
            if (drift) drift[(int64_t)t * H + h] = delta;
            s_mask[e] = m;
        }
    }
    __syncthreads();
    // per-token counts: counts = {full, partial, none, reused entries}
    unsigned long long full = 0, part = 0, none = 0, reused = 0;
    if (threadIdx.x < nt) {
        int c = 0;
        for (int h = 0; h < H; ++h) c += s_mask[threadIdx.x * H + h];
        reused = c;
        full = c == H;
        none = c == 0;
        part = !full && !none;
    }
    if (threadIdx.x < 32) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            full += __shfl_xor_sync(0xffffffffu, full, o);
            part += __shfl_xor_sync(0xffffffffu, part, o);
            none += __shfl_xor_sync(0xffffffffu, none, o);
            reused += __shfl_xor_sync(0xffffffffu, reused, o);
        }
        if (threadIdx.x == 0) {
            atomicAdd(counts + 0, full);
            atomicAdd(counts + 1, part);
            atomicAdd(counts + 2, none);
            atomicAdd(counts + 3, reused);
        }
    }
}

// ------------------------------------------------------------------------------ IRAP importance
constexpr int kIrapTile = 1024;     // keys per block of the main pass (256 threads x 4)
constexpr int kIrapRows = 128;      // query rows per block of the main pass

struct IrapGeom {
    int B, H, Sq, Sk, nkt, nqb;
};

// Row statistics of the contract normalisation: mode 1 (logits) -> (max, sum exp(x - max)) of
// the NaN-cleaned row; mode 2 (probabilities) -> (0, max(sum x, 1e-10)).  One warp per row.
__global__ void irap_rowstats_kernel(const float* __restrict__ x, int64_t rows, int Sk, int mode,
                                     float2* __restrict__ stats) {
    const int lane = threadIdx.x & 31;
    const int64_t r = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (r >= rows) return;
    const float* row = x + r * Sk;
    if (mode == 1) {
        float m = -FLT_MAX;
        for (int k = lane; k < Sk; k += 32) {
            float v = __ldg(row + k);
            v = v != v ? 0.0f : fminf(fmaxf(v, -FLT_MAX), FLT_MAX);
            m = fmaxf(m, v);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        double s = 0.0;
        for (int k = lane; k < Sk; k += 32) {
            float v = __ldg(row + k);
            v = v != v ? 0.0f : fminf(fmaxf(v, -FLT_MAX), FLT_MAX);
            s += (double)expf(v - m);
        }
        s = warp_sum_d(s);
        if (lane == 0) stats[r] = make_float2(m, (float)s);
    } else {
        double s = 0.0;
        for (int k = lane; k < Sk; k += 32) s += (double)__ldg(row + k);
        s = warp_sum_d(s);
        const float sf = (float)s;
        if (lane == 0) stats[r] = make_float2(0.0f, fmaxf(sf, 1e-10f));
    }
}

template <int MODE>
__device__ __forceinline__ float irap_weight(float x, float2 st) {
    if (MODE == 1) {
        x = x != x ? 0.0f : fminf(fmaxf(x, -FLT_MAX), FLT_MAX);
        x = __fdiv_rn(expf(x - st.x), st.y);
    } else if (MODE == 2) {
        x = __fdiv_rn(x, st.y);
    }
    // nan_to_num(nan=0, posinf=0, neginf=0): NaN fails the compare too
    return fabsf(x) < INFINITY ? x : 0.0f;
}

// log2 on the MUFU (inputs here are >= 1e-10: normal numbers, so flushing subnormals is moot)
__device__ __forceinline__ float lg2_approx(float x) {
    float y;
    asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Sums 8 values over the warp with 9 shuffles (a transpose-reduce butterfly): afterwards lane L
// holds the full sum of value ((L >> 4) & 1) * 4 + ((L >> 3) & 1) * 2 + ((L >> 2) & 1).
__device__ __forceinline__ float warp_sum8(float (&v)[8], int lane) {
    float a[4], b[2];
    const bool h16 = lane & 16, h8 = lane & 8, h4 = lane & 4;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float send = h16 ? v[i] : v[i + 4];
        const float keep = h16 ? v[i + 4] : v[i];
        a[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const float send = h8 ? a[i] : a[i + 2];
        const float keep = h8 ? a[i + 2] : a[i];
        b[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
    }
    float c = (h4 ? b[1] : b[0]) + __shfl_xor_sync(0xffffffffu, h4 ? b[0] : b[1], 4);
    c += __shfl_xor_sync(0xffffffffu, c, 2);
    c += __shfl_xor_sync(0xffffffffu, c, 1);
    return c;
}

// Four query rows (of one batch) of one thread's four keys: loads all four rows first, then
// folds each value into the column sums (compensated float32) and the rows' entropy terms.
// FULL: the block's whole key tile is in range and 16-byte aligned (no per-value checks).
template <int MODE, bool FULL>
__device__ __forceinline__ void irap_rows4(const float* __restrict__ row0, int64_t row_stride, int nr,
                                           const float2* __restrict__ st_row, int k0, int Sk, float (&col)[4],
                                           float (&comp)[4], float (&rc)[4], float (&rl)[4]) {
    constexpr int U = 4;
    float v[U][4];
    float2 st[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
        st[u] = make_float2(0.0f, 1.0f);
        if (u < nr) {
            const float* row = row0 + u * row_stride;
            if (MODE) st[u] = st_row[u];
            if (FULL) {
                const float4 a = __ldg(reinterpret_cast<const float4*>(row + k0));
                v[u][0] = a.x; v[u][1] = a.y; v[u][2] = a.z; v[u][3] = a.w;
            } else {
#pragma unroll
                for (int i = 0; i < 4; ++i) v[u][i] = k0 + i < Sk ? __ldg(row + k0 + i) : 0.0f;
            }
        }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
        if (u < nr) {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                if (FULL || k0 + i < Sk) {
                    const float w = irap_weight<MODE>(v[u][i], st[u]);
                    const float y = __fsub_rn(w, comp[i]);        // Kahan step: col += w
                    const float t = __fadd_rn(col[i], y);
                    comp[i] = __fsub_rn(__fsub_rn(t, col[i]), y);
                    col[i] = t;
                    const float c = fmaxf(w, 1e-10f);
                    rc[u] += c;
                    rl[u] = fmaf(c, lg2_approx(c), rl[u]);        // sum c log2 c; MUFU error ~2^-22
                }
            }
        }
    }
}

// grid (nkt, nqb, H), 256 threads: keys [kt*1024, +1024), query rows [qb*128, +128), all batches.
// colpart[(qb*H + h)*Sk + k] = sum over the block's rows of w (compensated float32 sum per
// column, one rounding to float64 per block); rowpart[(h*Sq + q)*nkt + kt] = (sum c, sum c ln c)
// over the block's keys and all batches.  Four query rows are loaded before any is reduced.
template <int MODE>
__global__ void __launch_bounds__(256, 4) irap_pass_kernel(const float* __restrict__ x, IrapGeom g,
                                                       const float2* __restrict__ stats, double* __restrict__ colpart,
                                                       double2* __restrict__ rowpart) {
    constexpr int U = 4;
    __shared__ double2 s_row[8][kIrapRows];
    const int kt = blockIdx.x, qb = blockIdx.y, h = blockIdx.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int k0 = kt * kIrapTile + threadIdx.x * 4;
    const int q0 = qb * kIrapRows;
    const int nq = min(kIrapRows, g.Sq - q0);
    const bool full = (g.Sk & 3) == 0 && (kt + 1) * kIrapTile <= g.Sk;
    float col[4] = {0.f, 0.f, 0.f, 0.f}, comp[4] = {0.f, 0.f, 0.f, 0.f};
    for (int qi = 0; qi < nq; qi += U) {
        const int nr = min(U, nq - qi);
        float rc[U] = {0.f, 0.f, 0.f, 0.f}, rl[U] = {0.f, 0.f, 0.f, 0.f};
        for (int b = 0; b < g.B; ++b) {
            const int64_t r = ((int64_t)b * g.H + h) * g.Sq + q0 + qi;      // first of the 4 rows
            const float* row0 = x + r * g.Sk;
            const float2* st_row = MODE ? stats + r : nullptr;
            if (full)
                irap_rows4<MODE, true>(row0, g.Sk, nr, st_row, k0, g.Sk, col, comp, rc, rl);
            else
                irap_rows4<MODE, false>(row0, g.Sk, nr, st_row, k0, g.Sk, col, comp, rc, rl);
        }
        // the 4 rows' (sum c, sum c log2 c) over the warp; value 2u is row u's sum c, 2u+1 its log sum
        float v8[8] = {rc[0], rl[0], rc[1], rl[1], rc[2], rl[2], rc[3], rl[3]};
        const float tot = warp_sum8(v8, lane);
        const int vi = ((lane >> 4) & 1) * 4 + ((lane >> 3) & 1) * 2 + ((lane >> 2) & 1);
        if ((lane & 3) == 0 && (vi >> 1) < nr) {
            double* slot = reinterpret_cast<double*>(&s_row[warp][qi + (vi >> 1)]);
            slot[vi & 1] = (double)tot * ((vi & 1) ? 0.69314718055994530942 : 1.0);   // log2 -> ln
        }
    }
    __syncthreads();
    for (int qi = threadIdx.x; qi < nq; qi += 256) {
        double a = 0.0, b = 0.0;
#pragma unroll
        for (int w = 0; w < 8; ++w) {
            a += s_row[w][qi].x;
            b += s_row[w][qi].y;
        }
        rowpart[((int64_t)h * g.Sq + q0 + qi) * g.nkt + kt] = make_double2(a, b);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i)
        if (k0 + i < g.Sk)
            colpart[((int64_t)qb * g.H + h) * g.Sk + k0 + i] = (double)col[i] - (double)comp[i];
}

// grid (ceil(Sk/256), H): received = sum / (B*Sq) -> EMA with the previous state; ema_hk [H,Sk]
// for the rank kernel, ema_out [Sk,H]; per-block delta_a partials (sum (ema-prev)^2, sum prev^2).
__global__ void irap_columns_kernel(const double* __restrict__ colpart, IrapGeom g, const float* __restrict__ prev,
                                    int S_prev, float d32, float e32, float* __restrict__ ema_hk,
                                    float* __restrict__ ema_out, double2* __restrict__ dparts) {
    __shared__ double s_a[8], s_b[8];
    const int h = blockIdx.y;
    const int k = blockIdx.x * blockDim.x + threadIdx.x;
    double da = 0.0, db = 0.0;
    if (k < g.Sk) {
        double s = 0.0;
        for (int qb = 0; qb < g.nqb; ++qb) s += colpart[((int64_t)qb * g.H + h) * g.Sk + k];
        const float received = (float)(s / ((double)g.B * (double)g.Sq));
        float ema = received;
        if (prev) {
            const float p = k < S_prev ? prev[(int64_t)k * g.H + h] : 0.0f;
            ema = __fadd_rn(__fmul_rn(d32, p), __fmul_rn(e32, received));
            const double df = (double)ema - (double)p;
            da = df * df;
            db = (double)p * (double)p;
        }
        ema_hk[(int64_t)h * g.Sk + k] = ema;
        ema_out[(int64_t)k * g.H + h] = ema;
    }
    da = warp_sum_d(da);
    db = warp_sum_d(db);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) {
        s_a[warp] = da;
        s_b[warp] = db;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        double a = 0.0, b = 0.0;
        for (int w = 0; w < (int)(blockDim.x >> 5); ++w) {
            a += s_a[w];
            b += s_b[w];
        }
        dparts[(int64_t)h * gridDim.x + blockIdx.x] = make_double2(a, b);
    }
}

// One block: the delta_a partials summed in a fixed order -> out[2].
__global__ void irap_dsum_kernel(const double2* __restrict__ dparts, int n, double* __restrict__ out) {
    __shared__ double s_a[32], s_b[32];
    double a = 0.0, b = 0.0;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        a += dparts[i].x;
        b += dparts[i].y;
    }
    a = warp_sum_d(a);
    b = warp_sum_d(b);
    if ((threadIdx.x & 31) == 0) {
        s_a[threadIdx.x >> 5] = a;
        s_b[threadIdx.x >> 5] = b;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        double x = 0.0, y = 0.0;
        for (int w = 0; w < (int)(blockDim.x >> 5); ++w) {
            x += s_a[w];
            y += s_b[w];
        }
        out[0] = x;
        out[1] = y;
    }
}

__device__ __forceinline__ float irap_blend(int rank, int i, const double2* __restrict__ rowpart, const IrapGeom& g,
                                           int h, double beta, float beta32, double layer_factor, double log_seq,
                                           int sink) {
    float nent = 0.0f;                               // no query row i: entropy term 0
    if (i < g.Sq) {
        double c = 0.0, l = 0.0;
        for (int kt = 0; kt < g.nkt; ++kt) {
            const double2 p = rowpart[((int64_t)h * g.Sq + i) * g.nkt + kt];
            c += p.x;
            l += p.y;
        }
        nent = (float)((log(c) - l / c) / log_seq);
    }
    const double rank_norm = ((double)rank + 1.0) / (double)g.Sk;
    double blended = __dmul_rn(1.0 - beta, rank_norm);
    blended = __dadd_rn(blended, (double)__fmul_rn(beta32, nent));
    const float imp = (float)fmin(__dmul_rn(blended, layer_factor), 1.0);
    return i < sink ? 1.0f : imp;
}

// grid (ceil(Sk/256), H): rank of each token's EMA within its head (ties by token index, a stable
// sort's order) by counting smaller keys over the whole head; then the blend:
// imp = min(((1-beta) * (rank+1)/Sk + f32(beta*entropy)) * layer_factor, 1), sinks forced to 1.
__global__ void __launch_bounds__(256) irap_rank_kernel(const float* __restrict__ ema_hk,
                                                       const double2* __restrict__ rowpart, IrapGeom g,
                                                       double beta, float beta32, double layer_factor,
                                                       double log_seq, int sink, float* __restrict__ importance) {
    __shared__ __align__(16) uint32_t s_key[2048];
    const int h = blockIdx.y;
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    const float* e = ema_hk + (int64_t)h * g.Sk;
    const uint32_t ki = i < g.Sk ? score_bits(e[i]) : 0u;
    // key j is below key i when kj < ki, or kj == ki and j < i: tokens before i count with <=,
    // tokens after i with <.  Keys are staged 2048 at a time and read 4 per shared load.
    int rank = 0;
    for (int j0 = 0; j0 < g.Sk; j0 += 2048) {
        const int n = min(2048, g.Sk - j0);
        __syncthreads();
        for (int j = threadIdx.x; j < 2048; j += blockDim.x) s_key[j] = j < n ? score_bits(e[j0 + j]) : 0xFFFFFFFFu;
        __syncthreads();
        if (i < g.Sk) {
            const int split = min(max(i - j0, 0), n);      // chunk positions [0, split) precede token i
            const uint4* k4 = reinterpret_cast<const uint4*>(s_key);
            int j = 0;
            for (; j + 4 <= (split & ~3); j += 4) {
                const uint4 q = k4[j >> 2];
                rank += (q.x <= ki) + (q.y <= ki) + (q.z <= ki) + (q.w <= ki);
            }
            for (; j < split; ++j) rank += s_key[j] <= ki;
            for (; j < n && (j & 3); ++j) rank += s_key[j] < ki;
            for (; j + 4 <= n; j += 4) {
                const uint4 q = k4[j >> 2];
                rank += (q.x < ki) + (q.y < ki) + (q.z < ki) + (q.w < ki);
            }
            for (; j < n; ++j) rank += s_key[j] < ki;
        }
    }
    if (i >= g.Sk) return;
    importance[(int64_t)i * g.H + h] = irap_blend(rank, i, rowpart, g, h, beta, beta32, layer_factor, log_seq, sink);
}

// One 1024-thread block per head for Sk <= kIrapSortMax: bitonic sort of the keys
// (order-preserving EMA bits << 32 | token: unique keys, so the sorted order is the stable
// order), then the token at sorted position p has rank p.  Thread t holds the E = N / 1024
// consecutive keys [t*E, t*E + E) in registers: exchange distances below E stay in the thread,
// those below 32*E go through warp shuffles, only the longer ones through shared memory.
constexpr int kIrapSortMax = 16384;

__device__ __forceinline__ unsigned long long bitonic_keep(unsigned long long a, unsigned long long b, int i, int k,
                                                           bool lower) {
    // position i keeps the smaller key when its run ascends and it is the lower of the pair
    const bool want_min = (((i & k) == 0) == lower);
    const bool a_small = a < b;
    return want_min ? (a_small ? a : b) : (a_small ? b : a);
}

template <int E>
__global__ void __launch_bounds__(1024) irap_sort_rank_kernel(const float* __restrict__ ema_hk,
                                                             const double2* __restrict__ rowpart, IrapGeom g,
                                                             double beta, float beta32, double layer_factor,
                                                             double log_seq, int sink, float* __restrict__ importance) {
    constexpr int N = 1024 * E;
    extern __shared__ unsigned long long s_keys[];   // [N]
    const int h = blockIdx.x, t = threadIdx.x, lane = t & 31;
    const float* e = ema_hk + (int64_t)h * g.Sk;
    unsigned long long x[E];
#pragma unroll
    for (int r = 0; r < E; ++r) {
        const int i = t * E + r;
        x[r] = i < g.Sk ? ((unsigned long long)score_bits(e[i]) << 32) | (unsigned)i : ~0ull;
    }
    for (int k = 2; k <= N; k <<= 1) {
        int j = k >> 1;
        for (; j >= E; j >>= 1) {
            if (j < 32 * E) {                              // partner in another lane of this warp
                const int lm = j / E;
#pragma unroll
                for (int r = 0; r < E; ++r) {
                    const int i = t * E + r;
                    const unsigned long long b = __shfl_xor_sync(0xffffffffu, x[r], lm);
                    x[r] = bitonic_keep(x[r], b, i, k, (lane & lm) == 0);
                }
            } else {                                       // partner in another warp
#pragma unroll
                for (int r = 0; r < E; ++r) s_keys[t * E + r] = x[r];
                __syncthreads();
#pragma unroll
                for (int r = 0; r < E; ++r) {
                    const int i = t * E + r;
                    x[r] = bitonic_keep(x[r], s_keys[i ^ j], i, k, (i & j) == 0);
                }
                __syncthreads();
            }
        }
        // the remaining distances j, j/2, ..., 1 (all < E): partners in this thread; the
        // distance is a compile-time constant so the keys stay in registers
#pragma unroll
        for (int jj = E / 2; jj > 0; jj >>= 1) {
            if (jj <= j) {
#pragma unroll
                for (int r = 0; r < E; ++r) {
                    if ((r ^ jj) > r) {
                        const int i = t * E + r;
                        const unsigned long long a = x[r], b = x[r ^ jj];
                        x[r] = bitonic_keep(a, b, i, k, true);
                        x[r ^ jj] = bitonic_keep(b, a, i ^ jj, k, false);
                    }
                }
            }
        }
    }
#pragma unroll
    for (int r = 0; r < E; ++r) {
        const int p = t * E + r;
        if (p < g.Sk) {
            const int i = (int)(x[r] & 0xFFFFFFFFu);
            importance[(int64_t)i * g.H + h] =
                irap_blend(p, i, rowpart, g, h, beta, beta32, layer_factor, log_seq, sink);
        }
    }
}

struct IrapScratch {
    size_t stats, colpart, rowpart, ema_hk, dparts, total;
};

static IrapScratch irap_layout(int B, int H, int Sq, int Sk) {
    const int nkt = (Sk + kIrapTile - 1) / kIrapTile, nqb = (Sq + kIrapRows - 1) / kIrapRows;
    const int ncb = (Sk + 255) / 256;
    auto up = [](size_t x) { return (x + 255) & ~(size_t)255; };
    IrapScratch s;
    size_t off = 0;
    s.stats = off;   off += up((size_t)B * H * Sq * sizeof(float2));
    s.colpart = off; off += up((size_t)nqb * H * Sk * sizeof(double));
    s.rowpart = off; off += up((size_t)H * Sq * nkt * sizeof(double2));
    s.ema_hk = off;  off += up((size_t)H * Sk * sizeof(float));
    s.dparts = off;  off += up((size_t)H * ncb * sizeof(double2));
    s.total = off;
    return s;
}

}  // namespace skv

using namespace skv;

extern "C" {

int skv_reuse_decide(const float* k_cur, const float* v_cur, const float* k_prev, const float* v_prev, int B, int H,
                     int S, int D, const float* importance, double effective_threshold, uint8_t* mask, float* drift,
                     int64_t* counts, void* stream) {
    if (!k_cur || !v_cur || !k_prev || !v_prev || !importance || !mask || !counts)
        return fail(SKV_ERR_INVALID_ARGUMENT, "reuse_decide: null pointer");
    if (B <= 0 || H <= 0 || S <= 0 || D <= 0) return fail(SKV_ERR_INVALID_ARGUMENT, "reuse_decide: bad size");
    if ((int64_t)kReuseTokens * H > 48 * 1024) return fail(SKV_ERR_TOO_LARGE, "reuse_decide: H too large");
    const uintptr_t a = reinterpret_cast<uintptr_t>(k_cur) | reinterpret_cast<uintptr_t>(v_cur) |
                        reinterpret_cast<uintptr_t>(k_prev) | reinterpret_cast<uintptr_t>(v_prev);
    if ((D & 3) == 0 && (a & 15) != 0) return fail(SKV_ERR_INVALID_ARGUMENT, "reuse_decide: K/V not 16-byte aligned");
    cudaStream_t st = as_stream(stream);
    if (cudaMemsetAsync(counts, 0, 4 * sizeof(int64_t), st) != cudaSuccess)
        return fail(SKV_ERR_CUDA, "reuse_decide: memset failed");
    const int blocks = (S + kReuseTokens - 1) / kReuseTokens;
    reuse_decide_kernel<<<blocks, 256, (size_t)kReuseTokens * H, st>>>(
        k_cur, v_cur, k_prev, v_prev, B, H, S, D, importance, effective_threshold, mask, drift,
        reinterpret_cast<unsigned long long*>(counts));
    return check_launch("reuse_decide");
}

size_t skv_irap_scratch_bytes(int B, int H, int Sq, int Sk) {
    if (B <= 0 || H <= 0 || Sq <= 0 || Sk <= 0) return 0;
    return irap_layout(B, H, Sq, Sk).total;
}

int skv_irap_importance(const float* scores, int B, int H, int Sq, int Sk, int input_mode, const float* ema_prev,
                        int S_prev, double irap_decay, double entropy_weight, int sink_tokens, double layer_factor,
                        void* scratch, size_t scratch_bytes, float* importance, float* ema, double* delta_parts,
                        void* stream) {
    if (!scores || !scratch || !importance || !ema || !delta_parts)
        return fail(SKV_ERR_INVALID_ARGUMENT, "irap_importance: null pointer");
    if (B <= 0 || H <= 0 || Sq <= 0 || Sk <= 0 || (ema_prev && S_prev < 0))
        return fail(SKV_ERR_INVALID_ARGUMENT, "irap_importance: bad size");
    if (input_mode < 0 || input_mode > 2) return fail(SKV_ERR_INVALID_ARGUMENT, "irap_importance: input mode %d", input_mode);
    if (!(irap_decay > 0.0 && irap_decay < 1.0)) return fail(SKV_ERR_INVALID_ARGUMENT, "irap_importance: irap_decay");
    if (!(entropy_weight >= 0.0 && entropy_weight <= 1.0))
        return fail(SKV_ERR_INVALID_ARGUMENT, "irap_importance: entropy_weight");
    if (sink_tokens < 0) return fail(SKV_ERR_INVALID_ARGUMENT, "irap_importance: sink_tokens");
    if (H > 65535 || (int64_t)(Sq + kIrapRows - 1) / kIrapRows > 65535)
        return fail(SKV_ERR_TOO_LARGE, "irap_importance: grid too large");
    if ((Sk & 3) == 0 && (reinterpret_cast<uintptr_t>(scores) & 15) != 0)
        return fail(SKV_ERR_INVALID_ARGUMENT, "irap_importance: scores not 16-byte aligned");
    const IrapScratch L = irap_layout(B, H, Sq, Sk);
    if (scratch_bytes < L.total) return fail(SKV_ERR_SCRATCH, "irap_importance: scratch %zu < %zu", scratch_bytes, L.total);
    uint8_t* sc = static_cast<uint8_t*>(scratch);
    float2* stats = reinterpret_cast<float2*>(sc + L.stats);
    double* colpart = reinterpret_cast<double*>(sc + L.colpart);
    double2* rowpart = reinterpret_cast<double2*>(sc + L.rowpart);
    float* ema_hk = reinterpret_cast<float*>(sc + L.ema_hk);
    double2* dparts = reinterpret_cast<double2*>(sc + L.dparts);
    IrapGeom g{B, H, Sq, Sk, (Sk + kIrapTile - 1) / kIrapTile, (Sq + kIrapRows - 1) / kIrapRows};
    cudaStream_t st = as_stream(stream);
    int rc;
    if (input_mode) {
        const int64_t rows = (int64_t)B * H * Sq;
        irap_rowstats_kernel<<<(unsigned)((rows * 32 + 255) / 256), 256, 0, st>>>(scores, rows, Sk, input_mode, stats);
        if ((rc = check_launch("irap_rowstats")) != SKV_OK) return rc;
    }
    const dim3 pgrid(g.nkt, g.nqb, H);
    if (input_mode == 0)
        irap_pass_kernel<0><<<pgrid, 256, 0, st>>>(scores, g, stats, colpart, rowpart);
    else if (input_mode == 1)
        irap_pass_kernel<1><<<pgrid, 256, 0, st>>>(scores, g, stats, colpart, rowpart);
    else
        irap_pass_kernel<2><<<pgrid, 256, 0, st>>>(scores, g, stats, colpart, rowpart);
    if ((rc = check_launch("irap_pass")) != SKV_OK) return rc;
    const int ncb = (Sk + 255) / 256;
    irap_columns_kernel<<<dim3(ncb, H), 256, 0, st>>>(colpart, g, ema_prev, S_prev, (float)irap_decay,
                                                       (float)(1.0 - irap_decay), ema_hk, ema, dparts);
    if ((rc = check_launch("irap_columns")) != SKV_OK) return rc;
    irap_dsum_kernel<<<1, 256, 0, st>>>(dparts, ncb * H, delta_parts);
    if ((rc = check_launch("irap_dsum")) != SKV_OK) return rc;
    const double log_seq = log((double)(Sk > 2 ? Sk : 2));
    if (Sk <= kIrapSortMax) {
        int E = 1;
        while (1024 * E < Sk) E <<= 1;
        const size_t smem = (size_t)1024 * E * sizeof(unsigned long long);
        if (smem > 48 * 1024) {
            static bool attr_set[64] = {};
            int devid = 0;
            cudaGetDevice(&devid);
            if (devid < 0 || devid >= 64) return fail(SKV_ERR_UNSUPPORTED, "irap_importance: device %d", devid);
            if (!attr_set[devid]) {
                if (cudaFuncSetAttribute(irap_sort_rank_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         8 * 1024 * 8) != cudaSuccess ||
                    cudaFuncSetAttribute(irap_sort_rank_kernel<16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         16 * 1024 * 8) != cudaSuccess)
                    return fail(SKV_ERR_CUDA, "irap_importance: shared memory attribute");
                attr_set[devid] = true;
            }
        }
        const double ew = entropy_weight;
        const float ew32 = (float)entropy_weight;
        switch (E) {
            case 1: irap_sort_rank_kernel<1><<<H, 1024, smem, st>>>(ema_hk, rowpart, g, ew, ew32, layer_factor, log_seq, sink_tokens, importance); break;
            case 2: irap_sort_rank_kernel<2><<<H, 1024, smem, st>>>(ema_hk, rowpart, g, ew, ew32, layer_factor, log_seq, sink_tokens, importance); break;
            case 4: irap_sort_rank_kernel<4><<<H, 1024, smem, st>>>(ema_hk, rowpart, g, ew, ew32, layer_factor, log_seq, sink_tokens, importance); break;
            case 8: irap_sort_rank_kernel<8><<<H, 1024, smem, st>>>(ema_hk, rowpart, g, ew, ew32, layer_factor, log_seq, sink_tokens, importance); break;
            default: irap_sort_rank_kernel<16><<<H, 1024, smem, st>>>(ema_hk, rowpart, g, ew, ew32, layer_factor, log_seq, sink_tokens, importance); break;
        }
    } else {
        irap_rank_kernel<<<dim3(ncb, H), 256, 0, st>>>(ema_hk, rowpart, g, entropy_weight, (float)entropy_weight,
                                                        layer_factor, log_seq, sink_tokens, importance);
    }
    return check_launch("irap_rank");
}

}  // extern "C"
