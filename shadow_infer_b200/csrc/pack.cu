// Fused gather + quantise + byte-pack, and unpack.
//
//  * skv_pack   -- PackedKVCache._do_pack_with_plan / _pack_int4_rows
//                  (shadowinfer/shadowkv/packed_kv_cache.py:222-388) with the quantisers of
//                  shadowinfer/utils/quantization.py:121-178, fused with the dense working
//                  copy of ShadowKVAgent._compress_kv_with_plan (shadowkv_agent.py:1698-1809).
//  * skv_unpack -- PackedKVCache.unpack / _dequantize_int4_bucket (packed_kv_cache.py:535-577,
//                  :636-656).
//
// Both walk K/V in memory order ([B,H,S,D] rows), so the fp32 side is streamed with 128-bit
// loads/stores; the per-entry slot (bucket position from the plan) locates the packed row.
// Lane layout of the vectorised kernels: every lane owns 16 consecutive values of a row
// (one int4 group at group size 16), D/16 lanes per row, 32/(D/16) rows per warp.  The
// int8 and int4 quantisers share one instruction stream (only the reduction width, the
// divisor and the final packing differ), so rows of both kinds in one warp do not diverge.
//
// Bit-exactness with the reference's torch CPU arithmetic: scale = IEEE amax/qmax (0 -> 1);
// q = clamp(rint(fl(x/scale))).  Each value is rounded from y = x * rcp(scale) with the
// 1.5*2^23 magic-number trick (round-half-even in the FP32 adder); a value whose y lies
// within 1e-4 of a .5 tie is recomputed with the exact IEEE division (|y - fl(x/scale)| is
// at most ~2.3e-5 for |y| <= 128, so elsewhere both round identically).  Packing uses
// cvt.pack.sat (int8: saturating s8; int4: saturating u4 of q + 8, high nibble first).
// Built without fast-math.
#include <string.h>

#include "skv_common.cuh"

namespace skv {

// ---------------------------------------------------------------------------------------
// 16-value lane helpers
// ---------------------------------------------------------------------------------------
__device__ __forceinline__ void ld16_stream(const float* p, float (&x)[16]) {
    const float4* q = reinterpret_cast<const float4*>(p);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float4 a = __ldcs(q + i);
        x[4 * i] = a.x;
        x[4 * i + 1] = a.y;
        x[4 * i + 2] = a.z;
        x[4 * i + 3] = a.w;
    }
}

__device__ __forceinline__ void st16(float* p, const float (&x)[16]) {
    float4* q = reinterpret_cast<float4*>(p);
#pragma unroll
    for (int i = 0; i < 4; ++i) q[i] = make_float4(x[4 * i], x[4 * i + 1], x[4 * i + 2], x[4 * i + 3]);
}

// Per-warp staging of RPW fp32 rows of D values (RPW*D*4 = 2 KB at D=128) in shared memory.
// 16-byte chunk c of a row lives at chunk c ^ ((c >> 2) & 7): the coalesced side (lane i ->
// chunk i + 32k) and the per-lane side (lane l of a row -> chunks 4l .. 4l+3) both touch 8
// distinct bank groups per 8 lanes, i.e. the 4-wavefront minimum per 512-byte access.
__device__ __forceinline__ int stage_chunk(int c) { return c ^ ((c >> 2) & 7); }

// Coalesced global -> staging copy of `rows` (<= RPW) contiguous rows starting at `src`.
template <int D, int RPW>
__device__ __forceinline__ void stage_in(float4* stage, const float* src, int rows, int lane) {
    constexpr int CPR = D / 4;                 // 16-byte chunks per row
    const float4* g = reinterpret_cast<const float4*>(src);
#pragma unroll
    for (int k = 0; k < RPW * CPR / 32; ++k) {
        const int q = lane + 32 * k;
        const int r = q / CPR, c = q % CPR;
        if (r < rows) stage[r * CPR + stage_chunk(c)] = __ldcs(g + q);
    }
}

template <int D, int RPW>
__device__ __forceinline__ void stage_out(const float4* stage, float* dst, int rows, int lane) {
    constexpr int CPR = D / 4;
    float4* g = reinterpret_cast<float4*>(dst);
#pragma unroll
    for (int k = 0; k < RPW * CPR / 32; ++k) {
        const int q = lane + 32 * k;
        const int r = q / CPR, c = q % CPR;
        if (r < rows) g[q] = stage[r * CPR + stage_chunk(c)];
    }
}

// The 16 values owned by lane l (chunks 4l .. 4l+3) of staged row r.
template <int D>
__device__ __forceinline__ void stage_get(const float4* stage, int r, int l, float (&x)[16]) {
    constexpr int CPR = D / 4;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const float4 a = stage[r * CPR + stage_chunk(4 * l + j)];
        x[4 * j] = a.x;
        x[4 * j + 1] = a.y;
        x[4 * j + 2] = a.z;
        x[4 * j + 3] = a.w;
    }
}

template <int D>
__device__ __forceinline__ void stage_put(float4* stage, int r, int l, const float (&x)[16]) {
    constexpr int CPR = D / 4;
#pragma unroll
    for (int j = 0; j < 4; ++j)
        stage[r * CPR + stage_chunk(4 * l + j)] = make_float4(x[4 * j], x[4 * j + 1], x[4 * j + 2], x[4 * j + 3]);
}

// d = (c << 16) | (sat_s8(a) << 8) | sat_s8(b)
__device__ __forceinline__ uint32_t pack_s8(int a, int b, uint32_t c) {
    uint32_t d;
    asm("cvt.pack.sat.s8.s32.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
// d = (c << 8) | (sat_u4(a) << 4) | sat_u4(b)
__device__ __forceinline__ uint32_t pack_u4(int a, int b, uint32_t c) {
    uint32_t d;
    asm("cvt.pack.sat.u4.s32.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

constexpr float kRoundMagic = 12582912.0f;   // 1.5 * 2^23: adding it rounds |y| < 2^22 to an integer

// max that propagates NaN (so a NaN deviation still sends the values to the exact path)
__device__ __forceinline__ float max_nan(float a, float b) {
    float d;
    asm("max.NaN.f32 %0, %1, %2;" : "=f"(d) : "f"(a), "f"(b));
    return d;
}

// q[i] = clamp(rint(fl(x[i] / s)), lo, hi) + OFF for 16 values; qf[i] = the rounded value without
// OFF.  OFF (8 for int4 nibbles) rides in the rounding constant: the integer part of
// y + 1.5*2^23 + OFF is rint(y) + OFF.  Values are rounded from the exact product y = x * rcp(s)
// (one fma with the constant), and the deviation y - rint(y) comes from a second fma; if any value
// lies within 1e-4 of a half-integer (or is not finite) all 16 take the exact IEEE division.  Away
// from ties rint(x * rcp(s)) == rint(fl(x / s)): the two differ by far less than 1e-4 for the
// |q| <= 128 range.  Out-of-range codes are clamped by the saturating packs that consume q.
template <int OFF>
__device__ __forceinline__ void quant16(const float (&x)[16], float s, float r, int lo, int hi, int (&q)[16],
                                        float (&qf)[16]) {
    constexpr float kM = kRoundMagic + (float)OFF;
    float dev = 0.0f;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        const float t = __fmaf_rn(x[i], r, kM);
        const float rf = __fsub_rn(t, kM);
        dev = max_nan(dev, fabsf(__fmaf_rn(x[i], r, -rf)));
        q[i] = __float_as_int(t) - 0x4B400000;
        qf[i] = rf;
    }
    if (!(dev < 0.4999f)) {
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            const int v = quant_value(x[i], s, lo, hi);
            q[i] = v + OFF;
            qf[i] = (float)v;
        }
    }
}

// ---------------------------------------------------------------------------------------
// pack
// ---------------------------------------------------------------------------------------
// One lane's 16 values of row (pos, b) into bucket `code`.  m_row / m_grp: absmax over the
// whole row and over this lane's int4 group (already reduced across lanes by the caller).
template <int LPR>
__device__ __forceinline__ void pack_lane(const float (&x)[16], int code, int64_t pos, int b, int B, int G,
                                          const skv_bucket& bb, bool is_v, float m_row, float m_grp,
                                          float (&dense)[16], int l) {
    constexpr int D = LPR * 16;
    const int64_t row = pos * B + b;
    void* payload = is_v ? bb.v : bb.k;
    float* scale = is_v ? bb.scale_v : bb.scale_k;
    if (code == 0) {
        st16(reinterpret_cast<float*>(payload) + row * D + l * 16, x);
#pragma unroll
        for (int i = 0; i < 16; ++i) dense[i] = x[i];
    } else if (code == 1) {
        uint32_t h[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const __half2 v = __floats2half2_rn(x[2 * i], x[2 * i + 1]);
            h[i] = *reinterpret_cast<const uint32_t*>(&v);
            const float2 f = __half22float2(v);
            dense[2 * i] = f.x;
            dense[2 * i + 1] = f.y;
        }
        uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<__half*>(payload) + row * D + l * 16);
        dst[0] = make_uint4(h[0], h[1], h[2], h[3]);
        dst[1] = make_uint4(h[4], h[5], h[6], h[7]);
    } else {
        // int8 (code 2) and int4 (code 3)
        const bool i4 = code == 3;
        const float s = quant_scale(i4 ? m_grp : m_row, i4 ? 7.0f : 127.0f);
        const float r = __frcp_rn(s);
        int q[16];
        if (i4) {
            quant16<8>(x, s, r, -8, 7, q, dense);         // q = code + 8, the stored nibble
            uint32_t w[2];
#pragma unroll
            for (int k = 0; k < 2; ++k) {
                uint32_t a = pack_u4(q[8 * k + 6], q[8 * k + 7], 0u);
                a = pack_u4(q[8 * k + 4], q[8 * k + 5], a);
                a = pack_u4(q[8 * k + 2], q[8 * k + 3], a);
                w[k] = pack_u4(q[8 * k], q[8 * k + 1], a);
            }
            const int64_t rb = (int64_t)B * D / 2;
            *reinterpret_cast<uint2*>(reinterpret_cast<uint8_t*>(payload) + pos * rb + (int64_t)b * (D / 2) + l * 8) =
                make_uint2(w[0], w[1]);
            const int lpg = G >> 4;   // lanes per int4 group
            if ((l & (lpg - 1)) == 0) scale[row * (D / G) + (l * 16) / G] = s;
        } else {
            quant16<0>(x, s, r, -128, 127, q, dense);
            uint32_t w[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) w[k] = pack_s8(q[4 * k + 1], q[4 * k], pack_s8(q[4 * k + 3], q[4 * k + 2], 0u));
            *reinterpret_cast<uint4*>(reinterpret_cast<int8_t*>(payload) + row * D + l * 16) =
                make_uint4(w[0], w[1], w[2], w[3]);
            if (l == 0) scale[row] = s;
        }
    }
}

// absmax of a lane's 16 values, reduced over its int4 group (m_grp) and its row (m_row).
// Every lane of the warp executes the shuffles, whatever its row's precision.
template <int LPR>
__device__ __forceinline__ void row_group_max(const float (&x)[16], int G, float& m_row, float& m_grp) {
    float m = 0.0f;
#pragma unroll
    for (int i = 0; i < 16; ++i) m = fmaxf(m, fabsf(x[i]));
    const int lpg = G >> 4;
    m_grp = m;
#pragma unroll
    for (int o = 1; o < LPR; o <<= 1) {
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        if ((o << 1) == lpg) m_grp = m;
    }
    m_row = m;
}

// Grid: x over (b, h), y over chunks of 8 warps * (32/LPR) rows.  A warp's RPW consecutive
// token rows of K and of V are contiguous in memory: they are fetched with coalesced 128-bit
// loads into the warp's staging buffer, then each lane quantises its 16 values, K first,
// then V (one tensor live at a time keeps the register count low).  DENSE adds the
// compress_kv working copy, staged back and stored coalesced.  DDESC: the bucket descriptors
// are read from device memory (`dbk`, written by pack_layout_kernel); a bucket without payload
// there (a slab that was too small) receives no stores.
template <int LPR, bool DENSE, bool DDESC = false>
__global__ void __launch_bounds__(256, 4) pack16_kernel(
    const float* __restrict__ k, const float* __restrict__ v, int B, int H, int S, int G,
    const int32_t* __restrict__ slot, Buckets bk, float* __restrict__ dense_k, float* __restrict__ dense_v,
    const float* __restrict__ k_prev, const float* __restrict__ v_prev, const uint8_t* __restrict__ reuse,
    const Buckets* __restrict__ dbk = nullptr) {
    constexpr int D = LPR * 16;
    constexpr int RPW = 32 / LPR;
    constexpr int CPR = D / 4;
    constexpr int kStageF4 = RPW * CPR;                   // float4s per staged tensor
    __shared__ float4 s_stage[8][2][kStageF4];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int l = lane % LPR, rsub = lane / LPR;
    const int bh = blockIdx.x;
    const int h = bh % H, b = bh / H;
    const int t0 = (blockIdx.y * 8 + warp) * RPW;
    if (t0 >= S) return;                                  // whole warp past the end
    const int rows = min(RPW, S - t0);
    const int t = t0 + rsub;
    const bool active = rsub < rows;
    const int64_t base = ((int64_t)bh * S + t0) * D;
    stage_in<D, RPW>(s_stage[warp][0], k + base, rows, lane);
    stage_in<D, RPW>(s_stage[warp][1], v + base, rows, lane);
    const int32_t sl = active ? slot[(int64_t)t * H + h] : -1;
    const bool from_prev = DENSE && active && reuse && k_prev && reuse[(int64_t)t * H + h];
    __syncwarp();
#pragma unroll 1
    for (int tensor = 0; tensor < 2; ++tensor) {
        float4* st = s_stage[warp][tensor];
        float x[16];
        if (active) {
            stage_get<D>(st, rsub, l, x);
        } else {
#pragma unroll
            for (int i = 0; i < 16; ++i) x[i] = 0.0f;
        }
        float mr, mg;
        row_group_max<LPR>(x, G, mr, mg);
        float dn[16];
        if (DDESC && active && sl >= 0) {
            const int code = slot_code(sl);
            const skv_bucket bc = dbk->b[code];
            if (bc.k) pack_lane<LPR>(x, code, slot_pos(sl), b, B, G, bc, tensor == 1, mr, mg, dn, l);
        } else if (active && sl >= 0) {
            const int code = slot_code(sl);
            pack_lane<LPR>(x, code, slot_pos(sl), b, B, G, bk.b[code], tensor == 1, mr, mg, dn, l);
        } else {
#pragma unroll
            for (int i = 0; i < 16; ++i) dn[i] = 0.0f;
        }
        if (DENSE) {
            float* dout = tensor ? dense_v : dense_k;
            __syncwarp();
            if (active && !from_prev) stage_put<D>(st, rsub, l, dn);
            __syncwarp();
            if (from_prev) {
                // reused rows come straight from the previous step's tensors
                const float* pin = tensor ? v_prev : k_prev;
                ld16_stream(pin + base + (int64_t)rsub * D + l * 16, dn);
                st16(dout + base + (int64_t)rsub * D + l * 16, dn);
            }
            const unsigned prev_rows = __ballot_sync(0xffffffffu, from_prev && l == 0);
            float4* g = reinterpret_cast<float4*>(dout + base);
#pragma unroll
            for (int kk = 0; kk < kStageF4 / 32; ++kk) {
                const int q = lane + 32 * kk;
                const int r = q / CPR, c = q % CPR;
                if (r < rows && !((prev_rows >> (r * LPR)) & 1u)) g[q] = st[r * CPR + stage_chunk(c)];
            }
        }
    }
}

// Generic path: one thread per (t,h) entry and tensor, any B, D and group.
__global__ void pack_generic_kernel(const float* __restrict__ k, const float* __restrict__ v, int B,
                                    int H, int S, int D, int G, const int32_t* __restrict__ slot,
                                    Buckets bk, float* __restrict__ dense_k, float* __restrict__ dense_v,
                                    const float* __restrict__ k_prev, const float* __restrict__ v_prev,
                                    const uint8_t* __restrict__ reuse) {
    const int64_t n = (int64_t)S * H;
    for (int64_t w = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; w < 2 * n;
         w += (int64_t)gridDim.x * blockDim.x) {
        const int which = (int)(w / n);  // 0: K, 1: V
        const int64_t e = w - which * n;
        const int64_t t = e / H, h = e - t * H;
        const float* src = which ? v : k;
        float* dense = which ? dense_v : dense_k;
        const float* prev = which ? v_prev : k_prev;
        const int32_t sl = slot[e];
        const int code = sl < 0 ? kCodeEvicted : slot_code(sl);
        const int64_t pos = sl < 0 ? 0 : slot_pos(sl);
        const bool use_prev = dense && reuse && prev && reuse[e];
        const skv_bucket* bb = code < kCodeEvicted ? &bk.b[code] : nullptr;
        void* payload = bb ? (which ? bb->v : bb->k) : nullptr;
        float* scale = bb ? (which ? bb->scale_v : bb->scale_k) : nullptr;
        const int NG = D / G;
        const int64_t rb = int4_row_bytes(B, D);
        for (int b = 0; b < B; ++b) {
            const float* x = src + (((int64_t)b * H + h) * S + t) * D;
            float* dn = dense ? dense + (((int64_t)b * H + h) * S + t) * D : nullptr;
            const float* pv = use_prev ? prev + (((int64_t)b * H + h) * S + t) * D : nullptr;
            const int64_t row = pos * B + b;
            if (code == 0) {
                float* o = reinterpret_cast<float*>(payload) + row * D;
                for (int d = 0; d < D; ++d) o[d] = x[d];
                if (dn) for (int d = 0; d < D; ++d) dn[d] = x[d];
            } else if (code == 1) {
                __half* o = reinterpret_cast<__half*>(payload) + row * D;
                for (int d = 0; d < D; ++d) {
                    o[d] = __float2half_rn(x[d]);
                    if (dn) dn[d] = __half2float(o[d]);
                }
            } else if (code == 2) {
                float m = 0.0f;
                for (int d = 0; d < D; ++d) m = fmaxf(m, fabsf(x[d]));
                const float s = quant_scale(m, 127.0f);
                scale[row] = s;
                int8_t* o = reinterpret_cast<int8_t*>(payload) + row * D;
                for (int d = 0; d < D; ++d) {
                    const int q = quant_value(x[d], s, -128, 127);
                    o[d] = (int8_t)q;
                    if (dn) dn[d] = (float)q;
                }
            } else if (code == 3) {
                uint8_t* o = reinterpret_cast<uint8_t*>(payload) + pos * rb;
                for (int g = 0; g < NG; ++g) {
                    float m = 0.0f;
                    for (int j = 0; j < G; ++j) m = fmaxf(m, fabsf(x[g * G + j]));
                    const float s = quant_scale(m, 7.0f);
                    scale[row * NG + g] = s;
                    for (int j = 0; j < G; ++j) {
                        const int d = g * G + j;
                        const int q = quant_value(x[d], s, -8, 7);
                        if (dn) dn[d] = (float)q;
                        const int64_t idx = (int64_t)b * D + d;  // nibble index in the entry row
                        const uint8_t nib = (uint8_t)(q + 8);
                        uint8_t& byte = o[idx >> 1];
                        if ((idx & 1) == 0) byte = (uint8_t)((byte & 0x0F) | (nib << 4));
                        else byte = (uint8_t)((byte & 0xF0) | (nib & 0x0F));
                    }
                }
                if (b == B - 1 && ((int64_t)B * D) % 2 == 1) {
                    uint8_t& last = o[rb - 1];
                    last = (uint8_t)((last & 0xF0) | 0x00);  // odd rows pad the low nibble with 0
                }
            } else if (dn) {
                for (int d = 0; d < D; ++d) dn[d] = 0.0f;
            }
            if (pv) for (int d = 0; d < D; ++d) dn[d] = pv[d];
        }
    }
}

// ---------------------------------------------------------------------------------------
// unpack
// ---------------------------------------------------------------------------------------
// One lane's 16 values of row (pos, b) of bucket `code`, dequantised exactly as the
// reference does (q.float() * scale).  Integer codes become floats through the exponent
// bits: 0x4B000000 | u is 2^23 + u.
template <int LPR>
__device__ __forceinline__ void unpack_lane(int code, int64_t pos, int b, int B, int G, const skv_bucket& bb,
                                            bool is_v, float (&y)[16], int l) {
    constexpr int D = LPR * 16;
    const int64_t row = pos * B + b;
    const void* payload = is_v ? bb.v : bb.k;
    const float* scale = is_v ? bb.scale_v : bb.scale_k;
    if (code == 0) {
        const float4* p = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(payload) + row * D + l * 16);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float4 a = p[i];
            y[4 * i] = a.x;
            y[4 * i + 1] = a.y;
            y[4 * i + 2] = a.z;
            y[4 * i + 3] = a.w;
        }
    } else if (code == 1) {
        const uint4* p = reinterpret_cast<const uint4*>(reinterpret_cast<const __half*>(payload) + row * D + l * 16);
        const uint4 a = p[0], c = p[1];
        const uint32_t w[8] = {a.x, a.y, a.z, a.w, c.x, c.y, c.z, c.w};
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
            y[2 * i] = f.x;
            y[2 * i + 1] = f.y;
        }
    } else if (code == 2) {
        const uint4 a = *reinterpret_cast<const uint4*>(reinterpret_cast<const int8_t*>(payload) + row * D + l * 16);
        const float s = scale[row];
        const uint32_t w[4] = {a.x ^ 0x80808080u, a.y ^ 0x80808080u, a.z ^ 0x80808080u, a.w ^ 0x80808080u};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            y[4 * i] = __fmul_rn(__fsub_rn(__int_as_float(__byte_perm(w[i], 0x4B000000u, 0x7540)), 8388736.0f), s);
            y[4 * i + 1] = __fmul_rn(__fsub_rn(__int_as_float(__byte_perm(w[i], 0x4B000000u, 0x7541)), 8388736.0f), s);
            y[4 * i + 2] = __fmul_rn(__fsub_rn(__int_as_float(__byte_perm(w[i], 0x4B000000u, 0x7542)), 8388736.0f), s);
            y[4 * i + 3] = __fmul_rn(__fsub_rn(__int_as_float(__byte_perm(w[i], 0x4B000000u, 0x7543)), 8388736.0f), s);
        }
    } else if (code == 3) {
        const int64_t rb = (int64_t)B * D / 2;
        const uint2 a = *reinterpret_cast<const uint2*>(reinterpret_cast<const uint8_t*>(payload) + pos * rb +
                                                        (int64_t)b * (D / 2) + l * 8);
        const float s = scale[row * (D / G) + (l * 16) / G];
        const uint32_t w[2] = {a.x, a.y};
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            const uint32_t hi = (w[k] >> 4) & 0x0F0F0F0Fu, lo = w[k] & 0x0F0F0F0Fu;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const uint32_t sel = 0x7540u | (uint32_t)j;
                y[8 * k + 2 * j] = __fmul_rn(__fsub_rn(__int_as_float(__byte_perm(hi, 0x4B000000u, sel)), 8388616.0f), s);
                y[8 * k + 2 * j + 1] =
                    __fmul_rn(__fsub_rn(__int_as_float(__byte_perm(lo, 0x4B000000u, sel)), 8388616.0f), s);
            }
        }
    } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) y[i] = 0.0f;
    }
}

template <int LPR>
__global__ void __launch_bounds__(256, 5) unpack16_kernel(Buckets bk, const int32_t* __restrict__ slot, int B, int H,
                                                          int S, int G, float* __restrict__ k_out,
                                                          float* __restrict__ v_out) {
    constexpr int D = LPR * 16;
    constexpr int RPW = 32 / LPR;
    constexpr int kStageF4 = RPW * D / 4;
    __shared__ float4 s_stage[8][kStageF4];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int l = lane % LPR, rsub = lane / LPR;
    // resident grid: each block walks (token chunk, b*h) items, b*h fastest -- the items in flight
    // cover every head of the same token range, whose bucket rows (token-major) are contiguous
    // (the host keeps the item count below 2^31)
    const int BH = B * H;
    const int items = BH * ((S + 8 * RPW - 1) / (8 * RPW));
    for (int it = blockIdx.x; it < items; it += gridDim.x) {
        const int bh = it % BH;
        const int h = bh % H, b = bh / H;
        const int t0 = ((it / BH) * 8 + warp) * RPW;
        if (t0 >= S) continue;
        const int rows = min(RPW, S - t0);
        const int t = t0 + rsub;
        const bool active = rsub < rows;
        const int32_t sl = active ? slot[(int64_t)t * H + h] : -1;
        const int code = sl < 0 ? kCodeEvicted : slot_code(sl);
        const int64_t pos = sl < 0 ? 0 : slot_pos(sl);
        const int64_t base = ((int64_t)bh * S + t0) * D;
        float4* st = s_stage[warp];
#pragma unroll 1
        for (int tensor = 0; tensor < 2; ++tensor) {
            float y[16];
            unpack_lane<LPR>(code, pos, b, B, G, bk.b[code < kCodeEvicted ? code : 0], tensor == 1, y, l);
            if (tensor) __syncwarp();        // the K rows have left the staging buffer
            if (active) stage_put<D>(st, rsub, l, y);
            __syncwarp();
            stage_out<D, RPW>(st, (tensor ? v_out : k_out) + base, rows, lane);
        }
        __syncwarp();        // the next item rewrites this warp's staging buffer
    }
}

__global__ void unpack_generic_kernel(Buckets bk, const int32_t* __restrict__ slot, int B, int H, int S,
                                      int D, int G, float* __restrict__ k_out, float* __restrict__ v_out) {
    const int64_t total = (int64_t)B * H * S * D;
    const int NG = D / G;
    const int64_t rb = int4_row_bytes(B, D);
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int d = (int)(i % D);
        const int64_t r = i / D;
        const int64_t t = r % S;
        const int64_t h = (r / S) % H;
        const int b = (int)(r / ((int64_t)S * H));
        const int32_t sl = slot[t * H + h];
        float yk = 0.0f, yv = 0.0f;
        if (sl >= 0) {
            const int code = slot_code(sl);
            const int64_t pos = slot_pos(sl);
            const skv_bucket& bb = bk.b[code];
            const int64_t row = pos * B + b;
            if (code == 0) {
                yk = reinterpret_cast<const float*>(bb.k)[row * D + d];
                yv = reinterpret_cast<const float*>(bb.v)[row * D + d];
            } else if (code == 1) {
                yk = __half2float(reinterpret_cast<const __half*>(bb.k)[row * D + d]);
                yv = __half2float(reinterpret_cast<const __half*>(bb.v)[row * D + d]);
            } else if (code == 2) {
                yk = __fmul_rn((float)reinterpret_cast<const int8_t*>(bb.k)[row * D + d], bb.scale_k[row]);
                yv = __fmul_rn((float)reinterpret_cast<const int8_t*>(bb.v)[row * D + d], bb.scale_v[row]);
            } else {
                const int64_t idx = (int64_t)b * D + d;
                const uint8_t ck = reinterpret_cast<const uint8_t*>(bb.k)[pos * rb + (idx >> 1)];
                const uint8_t cv = reinterpret_cast<const uint8_t*>(bb.v)[pos * rb + (idx >> 1)];
                const int nk = (idx & 1) ? (ck & 0x0F) : (ck >> 4);
                const int nv = (idx & 1) ? (cv & 0x0F) : (cv >> 4);
                yk = __fmul_rn((float)(nk - 8), bb.scale_k[row * NG + d / G]);
                yv = __fmul_rn((float)(nv - 8), bb.scale_v[row * NG + d / G]);
            }
        }
        k_out[i] = yk;
        v_out[i] = yv;
    }
}

// Vectorised kernels: D in {64, 128, 256} (D/16 lanes per row) and an int4 group that is a
// multiple of 16 values; other shapes take the generic kernels.
static int fast_lpr(int D, int G) {
    const int lpr = D == 64 ? 4 : (D == 128 ? 8 : (D == 256 ? 16 : 0));
    if (!lpr || G % 16) return 0;
    return lpr;
}

static bool is_aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// The vectorised kernels use 16-byte accesses on the fp32 side and row-aligned accesses on
// the bucket side; any pointer off a 16-byte boundary sends the call to the generic kernel.
static bool buckets_aligned(const skv_bucket* bk) {
    for (int p = 0; p < kNumBuckets; ++p) {
        if (bk[p].count == 0) continue;
        if (!is_aligned16(bk[p].k) || !is_aligned16(bk[p].v)) return false;
        if (bk[p].scale_k && (!is_aligned16(bk[p].scale_k) || !is_aligned16(bk[p].scale_v))) return false;
    }
    return true;
}

// Grid: x over (b, h), y over token chunks.  Blocks are issued x-fastest, so the blocks in
// flight cover every head of the same token range, whose bucket rows (token-major order)
// are contiguous: the packed side is then written / read sequentially.
static dim3 grid_rows(int B, int H, int S, int lpr) {
    const int rows_per_block = 8 * (32 / lpr);
    return dim3((unsigned)(B * H), (unsigned)((S + rows_per_block - 1) / rows_per_block));
}

// Resident blocks per SM of a 256-thread kernel (the launch-time occupancy).
template <typename Kernel>
static int resident_per_sm(Kernel kernel) {
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, 256, 0) != cudaSuccess || n < 1) n = 1;
    return n;
}

// Grid of the unpack kernels: one resident wave (per_sm blocks on every SM), each block walking
// its share of the (token chunk, b*h) items -- no block launch per 32-row chunk, no tail wave
// (63 -> 58 us on the cfg2 layer).  Pack keeps one block per chunk: its blocks hold 32 KB of
// staging and 64 registers per thread (4 per SM), and a block that walks items serialises their
// load latency (66 -> 70 us when looped).
static dim3 grid_items(int B, int H, int S, int lpr, int per_sm) {
    const int rows_per_block = 8 * (32 / lpr);
    const long long items = (long long)B * H * ((S + rows_per_block - 1) / rows_per_block);
    const long long resident = (long long)sm_count() * per_sm;
    return dim3((unsigned)(items < resident ? items : resident));
}

// Bucket layout of one allocation ("slab"), the same arithmetic on host and device: per
// precision in code order its k, v (and scale_k, scale_v) tensors in the reference layout,
// each starting on a 256-byte boundary.  Returns the slab bytes needed.
__host__ __device__ inline int64_t slab_layout(const int64_t* counts, int B, int D, int G, int64_t (*off)[4]) {
    int64_t total = 0;
    for (int c = 0; c < kNumBuckets; ++c) {
        const int64_t n = counts[c];
        int64_t nb[4] = {0, 0, 0, 0};
        if (c == 0) nb[0] = nb[1] = n * B * D * 4;
        else if (c == 1) nb[0] = nb[1] = n * B * D * 2;
        else if (c == 2) { nb[0] = nb[1] = n * B * D; nb[2] = nb[3] = n * B * 4; }
        else { nb[0] = nb[1] = n * ((B * D + 1) / 2); nb[2] = nb[3] = n * B * (D / G) * 4; }
        for (int t = 0; t < 4; ++t) {
            off[c][t] = -1;
            if (n == 0 || nb[t] == 0) continue;
            off[c][t] = total;
            total += (nb[t] + 255) / 256 * 256;
        }
    }
    return total;
}

// One thread: the descriptors of `slab` for the plan's device counts (bucket c's entries are
// flat_all[sum(counts[:c]) : +counts[c]]).  A slab smaller than the layout gets empty
// descriptors, and the pack kernel then writes nothing.
__global__ void pack_layout_kernel(const int64_t* __restrict__ counts, int B, int D, int G, uint8_t* slab,
                                   int64_t slab_bytes, const int64_t* flat_all, Buckets* __restrict__ out) {
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    int64_t cnt[kNumBuckets];
    for (int c = 0; c < kNumBuckets; ++c) cnt[c] = counts[c];
    int64_t off[kNumBuckets][4];
    const int64_t total = slab_layout(cnt, B, D, G, off);
    const bool fits = total <= slab_bytes;
    int64_t start = 0;
    for (int c = 0; c < kNumBuckets; ++c) {
        skv_bucket d;
        d.k = fits && off[c][0] >= 0 ? slab + off[c][0] : nullptr;
        d.v = fits && off[c][1] >= 0 ? slab + off[c][1] : nullptr;
        d.scale_k = fits && off[c][2] >= 0 ? reinterpret_cast<float*>(slab + off[c][2]) : nullptr;
        d.scale_v = fits && off[c][3] >= 0 ? reinterpret_cast<float*>(slab + off[c][3]) : nullptr;
        d.flat = const_cast<int64_t*>(flat_all) + start;
        d.count = fits ? cnt[c] : 0;
        out->b[c] = d;
        start += cnt[c];
    }
}

static int check_buckets(const skv_bucket* bk, const char* what) {
    if (!bk) return fail(SKV_ERR_INVALID_ARGUMENT, "%s: null bucket array", what);
    for (int p = 0; p < kNumBuckets; ++p) {
        if (bk[p].count < 0) return fail(SKV_ERR_INVALID_ARGUMENT, "%s: negative bucket count", what);
        if (bk[p].count > 0 && (!bk[p].k || !bk[p].v))
            return fail(SKV_ERR_INVALID_ARGUMENT, "%s: bucket %d has no payload", what, p);
        if (bk[p].count > 0 && p >= 2 && (!bk[p].scale_k || !bk[p].scale_v))
            return fail(SKV_ERR_INVALID_ARGUMENT, "%s: bucket %d has no scales", what, p);
    }
    return SKV_OK;
}

}  // namespace skv

using namespace skv;

extern "C" {

int skv_pack(const float* k, const float* v, int B, int H, int S, int D, int group_size,
             const int32_t* slot, const skv_bucket* buckets, float* dense_k, float* dense_v,
             const float* k_prev, const float* v_prev, const uint8_t* reuse_mask, void* stream) {
    if (B <= 0 || H <= 0 || S <= 0 || D <= 0) return fail(SKV_ERR_INVALID_ARGUMENT, "pack: bad shape");
    if (!k || !v || !slot) return fail(SKV_ERR_INVALID_ARGUMENT, "pack: null pointer");
    if ((dense_k == nullptr) != (dense_v == nullptr))
        return fail(SKV_ERR_INVALID_ARGUMENT, "pack: dense_k and dense_v must both be given");
    if ((k_prev == nullptr) != (v_prev == nullptr))
        return fail(SKV_ERR_INVALID_ARGUMENT, "pack: k_prev and v_prev must both be given");
    if ((int64_t)S * H > (int64_t(1) << 29)) return fail(SKV_ERR_TOO_LARGE, "pack: S*H above 2^29");
    int st = check_buckets(buckets, "pack");
    if (st) return st;
    if (group_size <= 0) return fail(SKV_ERR_GROUP_SIZE, "pack: group_size must be >= 1");
    const int G = int4_group(D, group_size);
    Buckets bk;
    for (int p = 0; p < kNumBuckets; ++p) bk.b[p] = buckets[p];
    cudaStream_t s = as_stream(stream);
    const bool aligned = is_aligned16(k) && is_aligned16(v) && is_aligned16(dense_k) && is_aligned16(dense_v) &&
                         is_aligned16(k_prev) && is_aligned16(v_prev) && buckets_aligned(buckets);
    const int lpr = aligned ? fast_lpr(D, G) : 0;
    if (lpr) {
        const dim3 grid = grid_rows(B, H, S, lpr);
#define SKV_PACK16(L, DN)                                                                                 \
    pack16_kernel<L, DN><<<grid, 256, 0, s>>>(k, v, B, H, S, G, slot, bk, dense_k, dense_v, k_prev, v_prev, \
                                              reuse_mask)
        if (dense_k) {
            if (lpr == 4) SKV_PACK16(4, true);
            else if (lpr == 8) SKV_PACK16(8, true);
            else SKV_PACK16(16, true);
        } else {
            if (lpr == 4) SKV_PACK16(4, false);
            else if (lpr == 8) SKV_PACK16(8, false);
            else SKV_PACK16(16, false);
        }
#undef SKV_PACK16
    } else {
        const int64_t n = 2 * (int64_t)S * H;
        const int64_t want = (n + 127) / 128;
        const int blocks = (int)(want < (int64_t)sm_count() * 16 ? want : (int64_t)sm_count() * 16);
        pack_generic_kernel<<<blocks, 128, 0, s>>>(k, v, B, H, S, D, G, slot, bk, dense_k, dense_v, k_prev, v_prev,
                                                   reuse_mask);
    }
    return check_launch("pack");
}

int64_t skv_pack_slab_bytes(const int64_t* counts, int B, int D, int group_size) {
    if (!counts || B <= 0 || D <= 0 || group_size <= 0) return -1;
    int64_t off[kNumBuckets][4];
    return slab_layout(counts, B, D, int4_group(D, group_size), off);
}

int skv_pack_slab(const float* k, const float* v, int B, int H, int S, int D, int group_size, const int32_t* slot,
                  const int64_t* counts, const int64_t* flat_all, void* slab, int64_t slab_bytes, void* desc,
                  void* stream) {
    if (B <= 0 || H <= 0 || S <= 0 || D <= 0 || slab_bytes < 0)
        return fail(SKV_ERR_INVALID_ARGUMENT, "pack_slab: bad shape or size");
    if (!k || !v || !slot || !counts || !flat_all || !slab || !desc)
        return fail(SKV_ERR_INVALID_ARGUMENT, "pack_slab: null pointer");
    if ((int64_t)S * H > (int64_t(1) << 29)) return fail(SKV_ERR_TOO_LARGE, "pack_slab: S*H above 2^29");
    if (group_size <= 0) return fail(SKV_ERR_GROUP_SIZE, "pack_slab: group_size must be >= 1");
    const int G = int4_group(D, group_size);
    const int lpr = fast_lpr(D, G);
    if (!lpr || !is_aligned16(k) || !is_aligned16(v) || (reinterpret_cast<uintptr_t>(slab) & 255) ||
        (reinterpret_cast<uintptr_t>(desc) & 15))
        return fail(SKV_ERR_UNSUPPORTED, "pack_slab: needs D in {64,128,256}, a group multiple of 16, 16-byte "
                                         "aligned K/V, a 256-byte aligned slab");
    cudaStream_t s = as_stream(stream);
    Buckets* dbk = reinterpret_cast<Buckets*>(desc);
    pack_layout_kernel<<<1, 32, 0, s>>>(counts, B, D, G, reinterpret_cast<uint8_t*>(slab), slab_bytes, flat_all, dbk);
    int st = check_launch("pack_slab layout");
    if (st) return st;
    Buckets none;
    memset(&none, 0, sizeof(none));
    const dim3 grid = grid_rows(B, H, S, lpr);
#define SKV_PACK16D(L)                                                                                          \
    pack16_kernel<L, false, true><<<grid, 256, 0, s>>>(k, v, B, H, S, G, slot, none, nullptr, nullptr, nullptr, \
                                                       nullptr, nullptr, dbk)
    if (lpr == 4) SKV_PACK16D(4);
    else if (lpr == 8) SKV_PACK16D(8);
    else SKV_PACK16D(16);
#undef SKV_PACK16D
    return check_launch("pack_slab");
}

int skv_unpack(const skv_bucket* buckets, const int32_t* slot, int B, int H, int S, int D, int int4_group,
               float* k_out, float* v_out, void* stream) {
    if (B <= 0 || H <= 0 || S <= 0 || D <= 0) return fail(SKV_ERR_INVALID_ARGUMENT, "unpack: bad shape");
    if (!slot || !k_out || !v_out) return fail(SKV_ERR_INVALID_ARGUMENT, "unpack: null pointer");
    int st = check_buckets(buckets, "unpack");
    if (st) return st;
    const int G = int4_group > 0 && D % int4_group == 0 ? int4_group : D;
    Buckets bk;
    for (int p = 0; p < kNumBuckets; ++p) bk.b[p] = buckets[p];
    cudaStream_t s = as_stream(stream);
    const bool aligned = is_aligned16(k_out) && is_aligned16(v_out) && buckets_aligned(buckets);
    const bool items_ok = (long long)B * H * ((S + 15) / 16) < (1ll << 31);   // 32-bit item index
    switch (aligned && items_ok ? fast_lpr(D, G) : 0) {
#define SKV_UNPACK16(L)                                                                                     \
    do {                                                                                                    \
        static const int per_sm = resident_per_sm(unpack16_kernel<L>);                                     \
        unpack16_kernel<L><<<grid_items(B, H, S, L, per_sm), 256, 0, s>>>(bk, slot, B, H, S, G, k_out, v_out); \
    } while (0)
        case 4: SKV_UNPACK16(4); break;
        case 8: SKV_UNPACK16(8); break;
        case 16:
            SKV_UNPACK16(16);
            break;
        default: {
            const int64_t total = (int64_t)B * H * S * D;
            const int64_t want = (total + 255) / 256;
            const int blocks = (int)(want < (int64_t)sm_count() * 16 ? want : (int64_t)sm_count() * 16);
            unpack_generic_kernel<<<blocks, 256, 0, s>>>(bk, slot, B, H, S, D, G, k_out, v_out);
        }
    }
#undef SKV_UNPACK16
    return check_launch("unpack");
}

}  // extern "C"
