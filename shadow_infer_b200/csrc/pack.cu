// Fused gather + quantise + byte-pack, and unpack.
//
//  * skv_pack   -- PackedKVCache._do_pack_with_plan / _pack_int4_rows
//                  (shadowinfer/shadowkv/packed_kv_cache.py:222-388) with the quantisers of
//                  shadowinfer/utils/quantization.py:121-178, fused with the dense working
//                  copy of ShadowKVAgent._compress_kv_with_plan (shadowkv_agent.py:1698-1809).
//  * skv_unpack -- PackedKVCache.unpack / _dequantize_int4_bucket (packed_kv_cache.py:535-577,
//                  :636-656).
//
// Both walk K/V in memory order ([B,H,S,D] rows, one warp per row of D floats), so the
// fp32 side is streamed with 128-bit loads/stores; the per-entry slot (bucket position
// from the plan) gives the packed side.  HBM-bound: a row costs 2*D*4 bytes of fp32 plus
// the packed row.  Quantisation is bit-exact with the reference's torch CPU arithmetic:
// IEEE division (no fast-math), round-half-even, clamp, nibble = q + 8, high nibble first.
#include "skv_common.cuh"

namespace skv {

template <int VEC>
struct Vec;
template <>
struct Vec<2> {
    static __device__ __forceinline__ void load(const float* p, float (&x)[2]) {
        const float2 a = __ldcs(reinterpret_cast<const float2*>(p));
        x[0] = a.x; x[1] = a.y;
    }
    static __device__ __forceinline__ void store(float* p, const float (&x)[2]) {
        *reinterpret_cast<float2*>(p) = make_float2(x[0], x[1]);
    }
};
template <>
struct Vec<4> {
    static __device__ __forceinline__ void load(const float* p, float (&x)[4]) {
        const float4 a = __ldcs(reinterpret_cast<const float4*>(p));
        x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
    }
    static __device__ __forceinline__ void store(float* p, const float (&x)[4]) {
        *reinterpret_cast<float4*>(p) = make_float4(x[0], x[1], x[2], x[3]);
    }
};
template <>
struct Vec<8> {
    static __device__ __forceinline__ void load(const float* p, float (&x)[8]) {
        const float4 a = __ldcs(reinterpret_cast<const float4*>(p));
        const float4 b = __ldcs(reinterpret_cast<const float4*>(p) + 1);
        x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
        x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
    }
    static __device__ __forceinline__ void store(float* p, const float (&x)[8]) {
        reinterpret_cast<float4*>(p)[0] = make_float4(x[0], x[1], x[2], x[3]);
        reinterpret_cast<float4*>(p)[1] = make_float4(x[4], x[5], x[6], x[7]);
    }
};

template <int N>
__device__ __forceinline__ void store_bytes(uint8_t* p, const uint8_t (&b)[N]) {
    if constexpr (N == 1) {
        p[0] = b[0];
    } else if constexpr (N == 2) {
        *reinterpret_cast<uint16_t*>(p) = (uint16_t)(b[0] | (b[1] << 8));
    } else if constexpr (N == 4) {
        *reinterpret_cast<uint32_t*>(p) =
            (uint32_t)b[0] | ((uint32_t)b[1] << 8) | ((uint32_t)b[2] << 16) | ((uint32_t)b[3] << 24);
    } else {
#pragma unroll
        for (int i = 0; i < N; i += 4) {
            *reinterpret_cast<uint32_t*>(p + i) = (uint32_t)b[i] | ((uint32_t)b[i + 1] << 8) |
                                                  ((uint32_t)b[i + 2] << 16) | ((uint32_t)b[i + 3] << 24);
        }
    }
}

template <int N>
__device__ __forceinline__ void load_bytes(const uint8_t* p, uint8_t (&b)[N]) {
    if constexpr (N == 1) {
        b[0] = p[0];
    } else if constexpr (N == 2) {
        const uint16_t w = *reinterpret_cast<const uint16_t*>(p);
        b[0] = w & 0xff; b[1] = w >> 8;
    } else {
#pragma unroll
        for (int i = 0; i < N; i += 4) {
            const uint32_t w = *reinterpret_cast<const uint32_t*>(p + i);
            b[i] = w & 0xff; b[i + 1] = (w >> 8) & 0xff; b[i + 2] = (w >> 16) & 0xff; b[i + 3] = w >> 24;
        }
    }
}

// Quantises one row slice (VEC values per lane, D = 32*VEC) into bucket `p` at entry `pos`,
// batch `b`; `dense` receives the compress_kv working-copy values.
template <int VEC>
__device__ __forceinline__ void pack_row(const float (&x)[VEC], int code, int64_t pos, int b, int B,
                                         int G, void* payload, float* scale, float (&dense)[VEC],
                                         int lane) {
    constexpr int D = 32 * VEC;
    const int64_t row = pos * B + b;
    if (code == 0) {
        Vec<VEC>::store(reinterpret_cast<float*>(payload) + row * D + lane * VEC, x);
#pragma unroll
        for (int j = 0; j < VEC; ++j) dense[j] = x[j];
    } else if (code == 1) {
        __half h[VEC];
#pragma unroll
        for (int j = 0; j < VEC; ++j) {
            h[j] = __float2half_rn(x[j]);
            dense[j] = __half2float(h[j]);
        }
        __half* dst = reinterpret_cast<__half*>(payload) + row * D + lane * VEC;
        if constexpr (VEC == 2) {
            *reinterpret_cast<__half2*>(dst) = __halves2half2(h[0], h[1]);
        } else {
#pragma unroll
            for (int j = 0; j < VEC; j += 4) {
                uint2 u;
                u.x = (uint32_t)__half_as_ushort(h[j]) | ((uint32_t)__half_as_ushort(h[j + 1]) << 16);
                u.y = (uint32_t)__half_as_ushort(h[j + 2]) | ((uint32_t)__half_as_ushort(h[j + 3]) << 16);
                *reinterpret_cast<uint2*>(dst + j) = u;
            }
        }
    } else if (code == 2) {
        float m = 0.0f;
#pragma unroll
        for (int j = 0; j < VEC; ++j) m = fmaxf(m, fabsf(x[j]));
        m = warp_max(m);
        const float s = quant_scale(m, 127.0f);
        const float r = __frcp_rn(s);
        uint8_t q[VEC];
#pragma unroll
        for (int j = 0; j < VEC; ++j) {
            const int v = quant_value_fast(x[j], s, r, -128, 127);
            q[j] = (uint8_t)(int8_t)v;
            dense[j] = (float)v;
        }
        store_bytes<VEC>(reinterpret_cast<uint8_t*>(payload) + row * D + lane * VEC, q);
        if (lane == 0) scale[row] = s;
    } else if (code == 3) {
        // the fast path requires the group to span a power-of-two number of whole lanes
        const int NG = D / G;
        float m = 0.0f;
#pragma unroll
        for (int j = 0; j < VEC; ++j) m = fmaxf(m, fabsf(x[j]));
        const int L = G / VEC;
        m = group_max(m, L);
        const float s = quant_scale(m, 7.0f);
        const float r = __frcp_rn(s);
        if ((lane & (L - 1)) == 0) scale[row * NG + (lane * VEC) / G] = s;
        uint8_t bytes[VEC / 2];
#pragma unroll
        for (int j = 0; j < VEC; j += 2) {
            const int q0 = quant_value_fast(x[j], s, r, -8, 7);
            const int q1 = quant_value_fast(x[j + 1], s, r, -8, 7);
            dense[j] = (float)q0;
            dense[j + 1] = (float)q1;
            bytes[j / 2] = (uint8_t)(((q0 + 8) << 4) | ((q1 + 8) & 0x0F));
        }
        const int64_t rb = (int64_t)B * D / 2;
        store_bytes<VEC / 2>(reinterpret_cast<uint8_t*>(payload) + pos * rb + (int64_t)b * (D / 2) +
                                 lane * (VEC / 2),
                             bytes);
    } else {
#pragma unroll
        for (int j = 0; j < VEC; ++j) dense[j] = 0.0f;
    }
}

// Grid: x over token chunks of 8 warps * RPW rows, y over (b, h).  Each warp loads all
// of its RPW K and V rows (128-bit streaming loads) before quantising any of them.
template <int VEC, int RPW>
__global__ void __launch_bounds__(256) pack_fast_kernel(
    const float* __restrict__ k, const float* __restrict__ v, int B, int H, int S, int G,
    const int32_t* __restrict__ slot, Buckets bk, float* __restrict__ dense_k,
    float* __restrict__ dense_v, const float* __restrict__ k_prev, const float* __restrict__ v_prev,
    const uint8_t* __restrict__ reuse) {
    constexpr int D = 32 * VEC;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int bh = blockIdx.y;
    const int h = bh % H, b = bh / H;
    const int t0 = (blockIdx.x * 8 + warp) * RPW;
    if (t0 >= S) return;
    const int64_t base = (int64_t)bh * S * D + lane * VEC;
    float xk[RPW][VEC], xv[RPW][VEC];
    int32_t sl[RPW];
#pragma unroll
    for (int i = 0; i < RPW; ++i) {
        const int t = t0 + i;
        if (t < S) {
            Vec<VEC>::load(k + base + (int64_t)t * D, xk[i]);
            Vec<VEC>::load(v + base + (int64_t)t * D, xv[i]);
            sl[i] = slot[t * H + h];
        }
    }
#pragma unroll
    for (int i = 0; i < RPW; ++i) {
        const int t = t0 + i;
        if (t >= S) break;
        const int code = sl[i] < 0 ? kCodeEvicted : slot_code(sl[i]);
        const int64_t pos = sl[i] < 0 ? 0 : slot_pos(sl[i]);
        float dk[VEC], dv[VEC];
        if (code < kCodeEvicted) {
            const skv_bucket& bb = bk.b[code];
            pack_row<VEC>(xk[i], code, pos, b, B, G, bb.k, bb.scale_k, dk, lane);
            pack_row<VEC>(xv[i], code, pos, b, B, G, bb.v, bb.scale_v, dv, lane);
        } else {
#pragma unroll
            for (int j = 0; j < VEC; ++j) dk[j] = dv[j] = 0.0f;
        }
        if (dense_k) {
            const int64_t off = base + (int64_t)t * D;
            if (reuse && k_prev && reuse[(int64_t)t * H + h]) {
                Vec<VEC>::load(k_prev + off, dk);
                Vec<VEC>::load(v_prev + off, dv);
            }
            Vec<VEC>::store(dense_k + off, dk);
            Vec<VEC>::store(dense_v + off, dv);
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
template <int VEC>
__device__ __forceinline__ void unpack_row(int code, int64_t pos, int b, int B, int G,
                                           const void* payload, const float* scale, float (&y)[VEC],
                                           int lane) {
    constexpr int D = 32 * VEC;
    const int64_t row = pos * B + b;
    if (code == 0) {
        Vec<VEC>::load(reinterpret_cast<const float*>(payload) + row * D + lane * VEC, y);
    } else if (code == 1) {
        const __half* src = reinterpret_cast<const __half*>(payload) + row * D + lane * VEC;
        if constexpr (VEC == 2) {
            const __half2 h2 = *reinterpret_cast<const __half2*>(src);
            y[0] = __low2float(h2);
            y[1] = __high2float(h2);
        } else {
#pragma unroll
            for (int j = 0; j < VEC; j += 4) {
                const uint2 u = *reinterpret_cast<const uint2*>(src + j);
                y[j] = __half2float(__ushort_as_half((unsigned short)(u.x & 0xffff)));
                y[j + 1] = __half2float(__ushort_as_half((unsigned short)(u.x >> 16)));
                y[j + 2] = __half2float(__ushort_as_half((unsigned short)(u.y & 0xffff)));
                y[j + 3] = __half2float(__ushort_as_half((unsigned short)(u.y >> 16)));
            }
        }
    } else if (code == 2) {
        uint8_t q[VEC];
        load_bytes<VEC>(reinterpret_cast<const uint8_t*>(payload) + row * D + lane * VEC, q);
        const float s = scale[row];
#pragma unroll
        for (int j = 0; j < VEC; ++j) y[j] = __fmul_rn((float)(int8_t)q[j], s);
    } else if (code == 3) {
        const int NG = D / G;
        const int64_t rb = (int64_t)B * D / 2;
        uint8_t bytes[VEC / 2];
        load_bytes<VEC / 2>(reinterpret_cast<const uint8_t*>(payload) + pos * rb + (int64_t)b * (D / 2) +
                                lane * (VEC / 2),
                            bytes);
        if (G >= VEC) {
            const float s0 = scale[row * NG + (lane * VEC) / G];
#pragma unroll
            for (int j = 0; j < VEC; j += 2) {
                y[j] = __fmul_rn((float)((int)(bytes[j / 2] >> 4) - 8), s0);
                y[j + 1] = __fmul_rn((float)((int)(bytes[j / 2] & 0x0F) - 8), s0);
            }
        } else {
#pragma unroll
            for (int j = 0; j < VEC; j += 2) {
                const float s0 = scale[row * NG + (lane * VEC + j) / G];
                const float s1 = scale[row * NG + (lane * VEC + j + 1) / G];
                y[j] = __fmul_rn((float)((int)(bytes[j / 2] >> 4) - 8), s0);
                y[j + 1] = __fmul_rn((float)((int)(bytes[j / 2] & 0x0F) - 8), s1);
            }
        }
    } else {
#pragma unroll
        for (int j = 0; j < VEC; ++j) y[j] = 0.0f;
    }
}

// Raw bytes of one lane's slice of a packed row (VEC values), fetched before decoding so a
// warp keeps all of its rows' loads in flight at once.
template <int VEC>
struct RawSlice {
    uint32_t w[VEC];   // fp32: VEC words; fp16: VEC/2; int8: VEC/4 (or 1 sub-word); int4: VEC/8 (or 1 sub-word)
    float s;           // int8 row scale / int4 group scale
};

template <int VEC>
__device__ __forceinline__ void load_raw(int code, int64_t pos, int b, int B, int G, const void* payload,
                                         const float* scale, RawSlice<VEC>& r, int lane) {
    constexpr int D = 32 * VEC;
    const int64_t row = pos * B + b;
    if (code == 0) {
        const uint32_t* p = reinterpret_cast<const uint32_t*>(payload) + row * D + lane * VEC;
        if constexpr (VEC == 2) {
            const uint2 a = *reinterpret_cast<const uint2*>(p);
            r.w[0] = a.x; r.w[1] = a.y;
        } else {
#pragma unroll
            for (int j = 0; j < VEC; j += 4) {
                const uint4 a = *reinterpret_cast<const uint4*>(p + j);
                r.w[j] = a.x; r.w[j + 1] = a.y; r.w[j + 2] = a.z; r.w[j + 3] = a.w;
            }
        }
    } else if (code == 1) {
        const uint16_t* p = reinterpret_cast<const uint16_t*>(payload) + row * D + lane * VEC;
        if constexpr (VEC == 2) {
            r.w[0] = *reinterpret_cast<const uint32_t*>(p);
        } else {
#pragma unroll
            for (int j = 0; j < VEC / 2; j += 2) {
                const uint2 a = *reinterpret_cast<const uint2*>(p + 2 * j);
                r.w[j] = a.x; r.w[j + 1] = a.y;
            }
        }
    } else if (code == 2) {
        const uint8_t* p = reinterpret_cast<const uint8_t*>(payload) + row * D + lane * VEC;
        if constexpr (VEC == 2) r.w[0] = *reinterpret_cast<const uint16_t*>(p);
        else if constexpr (VEC == 4) r.w[0] = *reinterpret_cast<const uint32_t*>(p);
        else { const uint2 a = *reinterpret_cast<const uint2*>(p); r.w[0] = a.x; r.w[1] = a.y; }
        r.s = scale[row];
    } else {
        const int64_t rb = (int64_t)B * D / 2;
        const uint8_t* p = reinterpret_cast<const uint8_t*>(payload) + pos * rb + (int64_t)b * (D / 2) + lane * (VEC / 2);
        if constexpr (VEC == 2) r.w[0] = *p;
        else if constexpr (VEC == 4) r.w[0] = *reinterpret_cast<const uint16_t*>(p);
        else r.w[0] = *reinterpret_cast<const uint32_t*>(p);
        const int NG = D / G;
        r.s = scale[row * NG + (lane * VEC) / G];
    }
}

// Decodes a RawSlice; int4 requires G >= VEC (one group scale per lane).
template <int VEC>
__device__ __forceinline__ void decode_raw(int code, const RawSlice<VEC>& r, float (&y)[VEC]) {
    if (code == 0) {
#pragma unroll
        for (int j = 0; j < VEC; ++j) y[j] = __uint_as_float(r.w[j]);
    } else if (code == 1) {
#pragma unroll
        for (int j = 0; j < VEC; j += 2) {
            y[j] = __half2float(__ushort_as_half((unsigned short)(r.w[j / 2] & 0xffff)));
            y[j + 1] = __half2float(__ushort_as_half((unsigned short)(r.w[j / 2] >> 16)));
        }
    } else if (code == 2) {
#pragma unroll
        for (int j = 0; j < VEC; ++j) {
            const int8_t q = (int8_t)((r.w[j / 4] >> (8 * (j % 4))) & 0xff);
            y[j] = __fmul_rn((float)q, r.s);
        }
    } else if (code == 3) {
#pragma unroll
        for (int j = 0; j < VEC; j += 2) {
            const uint32_t byte = (r.w[(j / 2) / 4] >> (8 * ((j / 2) % 4))) & 0xff;
            y[j] = __fmul_rn((float)((int)(byte >> 4) - 8), r.s);
            y[j + 1] = __fmul_rn((float)((int)(byte & 0x0F) - 8), r.s);
        }
    } else {
#pragma unroll
        for (int j = 0; j < VEC; ++j) y[j] = 0.0f;
    }
}

template <int VEC, int RPW>
__global__ void __launch_bounds__(256) unpack_fast_kernel(Buckets bk, const int32_t* __restrict__ slot,
                                                          int B, int H, int S, int G,
                                                          float* __restrict__ k_out,
                                                          float* __restrict__ v_out) {
    constexpr int D = 32 * VEC;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int bh = blockIdx.y;
    const int h = bh % H, b = bh / H;
    const int t0 = (blockIdx.x * 8 + warp) * RPW;
    if (t0 >= S) return;
    const int64_t base = (int64_t)bh * S * D + lane * VEC;
    int32_t sl[RPW];
#pragma unroll
    for (int i = 0; i < RPW; ++i) sl[i] = (t0 + i < S) ? slot[(t0 + i) * H + h] : -1;
    RawSlice<VEC> rk[RPW], rv[RPW];
#pragma unroll
    for (int i = 0; i < RPW; ++i) {
        const int code = sl[i] < 0 ? kCodeEvicted : slot_code(sl[i]);
        if (code < kCodeEvicted) {
            const int64_t pos = slot_pos(sl[i]);
            const skv_bucket& bb = bk.b[code];
            load_raw<VEC>(code, pos, b, B, G, bb.k, bb.scale_k, rk[i], lane);
            load_raw<VEC>(code, pos, b, B, G, bb.v, bb.scale_v, rv[i], lane);
        }
    }
#pragma unroll
    for (int i = 0; i < RPW; ++i) {
        const int t = t0 + i;
        if (t >= S) break;
        const int code = sl[i] < 0 ? kCodeEvicted : slot_code(sl[i]);
        float yk[VEC], yv[VEC];
        decode_raw<VEC>(code, rk[i], yk);
        decode_raw<VEC>(code, rv[i], yv);
        Vec<VEC>::store(k_out + base + (int64_t)t * D, yk);
        Vec<VEC>::store(v_out + base + (int64_t)t * D, yv);
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

// The warp-per-row kernels cover D = 32*VEC with VEC in {2,4,8} and an int4 group that spans a
// power-of-two number of whole lanes (group 16 at D = 64/128/256); other shapes take the
// generic kernels.
static int fast_vec_unpack(int D, int G) {
    const int vec = D == 64 ? 2 : (D == 128 ? 4 : (D == 256 ? 8 : 0));
    if (!vec || G < vec || G % vec) return 0;
    const int L = G / vec;
    return (L <= 32 && (L & (L - 1)) == 0) ? vec : 0;
}

static int fast_vec(int D, int G) { return fast_vec_unpack(D, G); }

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

constexpr int kPackRPW = 2;
constexpr int kUnpackRPW = 4;

static dim3 grid_2d(int B, int H, int S, int rpw) {
    return dim3((unsigned)((S + 8 * rpw - 1) / (8 * rpw)), (unsigned)(B * H));
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
    switch (aligned ? fast_vec(D, G) : 0) {
        case 2:
            pack_fast_kernel<2, kPackRPW><<<grid_2d(B, H, S, kPackRPW), 256, 0, s>>>(
                k, v, B, H, S, G, slot, bk, dense_k, dense_v, k_prev, v_prev, reuse_mask);
            break;
        case 4:
            pack_fast_kernel<4, kPackRPW><<<grid_2d(B, H, S, kPackRPW), 256, 0, s>>>(
                k, v, B, H, S, G, slot, bk, dense_k, dense_v, k_prev, v_prev, reuse_mask);
            break;
        case 8:
            pack_fast_kernel<8, kPackRPW><<<grid_2d(B, H, S, kPackRPW), 256, 0, s>>>(
                k, v, B, H, S, G, slot, bk, dense_k, dense_v, k_prev, v_prev, reuse_mask);
            break;
        default: {
            const int64_t n = 2 * (int64_t)S * H;
            const int64_t want = (n + 127) / 128;
            const int blocks = (int)(want < (int64_t)sm_count() * 16 ? want : (int64_t)sm_count() * 16);
            pack_generic_kernel<<<blocks, 128, 0, s>>>(k, v, B, H, S, D, G, slot, bk, dense_k, dense_v,
                                                       k_prev, v_prev, reuse_mask);
        }
    }
    return check_launch("pack");
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
    switch (aligned ? fast_vec_unpack(D, G) : 0) {
        case 2:
            unpack_fast_kernel<2, kUnpackRPW><<<grid_2d(B, H, S, kUnpackRPW), 256, 0, s>>>(bk, slot, B, H, S, G,
                                                                                            k_out, v_out);
            break;
        case 4:
            unpack_fast_kernel<4, kUnpackRPW><<<grid_2d(B, H, S, kUnpackRPW), 256, 0, s>>>(bk, slot, B, H, S, G,
                                                                                            k_out, v_out);
            break;
        case 8:
            unpack_fast_kernel<8, kUnpackRPW><<<grid_2d(B, H, S, kUnpackRPW), 256, 0, s>>>(bk, slot, B, H, S, G,
                                                                                            k_out, v_out);
            break;
        default: {
            const int64_t total = (int64_t)B * H * S * D;
            const int64_t want = (total + 255) / 256;
            const int blocks = (int)(want < (int64_t)sm_count() * 16 ? want : (int64_t)sm_count() * 16);
            unpack_generic_kernel<<<blocks, 256, 0, s>>>(bk, slot, B, H, S, D, G, k_out, v_out);
        }
    }
    return check_launch("unpack");
}

}  // extern "C"
