// Attention read directly from the packed cache, on the sm_100a tensor cores.
//
// Oracle: PackedKVCache.unpack() (shadowinfer/shadowkv/packed_kv_cache.py:535-577) followed by
// the dense, non-causal attention of SimpleDiffusionLLM._compute_block
// (shadowinfer/models/simple_diffusion_llm.py:165-169): O = softmax(Q K^T / sqrt(D)) V with
// evicted (t,h) entries present as ZERO rows of K and V (logit 0, no value).
//
// skv_head_index   -- per head, the stored entries of the cache grouped by precision (token
//                     order inside a group): the KV row list the attention kernel walks.
// skv_packed_attention -- one CTA per (128-query tile, head, batch), warp-specialised:
//   warps 0-3  softmax: thread i owns query row i = TMEM lane i; reads S from TMEM, keeps the
//              running max / sum (lazy rescale of O when the max grows by more than 2^8),
//              writes P (fp16) into shared memory, finally normalises O and stores it.
//   warps 4-7  converters: fetch packed K/V rows straight from the buckets and write fp16 tiles
//              in the 128B-swizzled UMMA layout (fp32 -> fp16 RNE; fp16 copied; int8 codes
//              converted EXACTLY and their per-row scales folded into the softmax: K scale
//              into the logit factor, V scale into P; int4 dequantised in fp32 then rounded).
//   warp 8     MMA issuer: S_j = Q K_j^T into one of two TMEM S buffers, O += P_j V_j into the
//              TMEM O accumulator (tcgen05.mma kind::f16, M=128, fp32 accumulate), completion
//              signalled with tcgen05.commit on mbarriers.
// Evicted entries never enter a tile: their contribution (count * 2^(0 - m)) is added to the
// softmax denominator analytically.  Every mbarrier wait is bounded; a timeout sets the error
// word and all roles drain to the final barrier before TMEM is released.
#include <math.h>
#include <string.h>

#include "skv_common.cuh"
#include "sm100_ptx.cuh"

namespace skv {
using namespace sm100;

constexpr int kBM = 128;          // queries per CTA
constexpr int kBN = 128;          // KV rows per tile
constexpr int kStages = 2;        // K/V tile stages in shared memory
constexpr int kSoftmaxWarps = 4;
constexpr int kConvWarps = 8;
constexpr int kAttnThreads = (kSoftmaxWarps + kConvWarps + 1) * 32;
constexpr uint32_t kTmemCols = 512;
constexpr float kRescaleThreshold = 8.0f;   // log2 units

enum AttnError { kErrNone = 0, kErrKvFull = 1, kErrKvEmpty = 2, kErrSFull = 3, kErrPFull = 4, kErrPvDone = 5,
                 kErrDrain = 6 };

template <int D>
struct AttnLayout {
    static constexpr int NA = D / 64;                   // 128-byte swizzle atoms per row
    static constexpr int kAtomQ = kBM * 128;            // bytes of one atom column of a 128-row tile
    static constexpr int kQ = 0;
    static constexpr int kK = kQ + NA * kAtomQ;
    static constexpr int kV = kK + kStages * NA * kBN * 128;
    static constexpr int kP = kV + kStages * NA * kBN * 128;
    static constexpr int kEnt = kP + 2 * kBM * 128;     // P: K-dim = kBN = 128 -> 2 atoms
    static constexpr int kBar = kEnt + kStages * kBN * 4;   // per-stage entry (slot) lists
    static constexpr int kNumBars = 2 * kStages + 2 + 1 + 1 + 1;
    static constexpr int kTmemSlot = kBar + kNumBars * 8;
    static constexpr int kBytes = kTmemSlot + 16;
    // + slack to align the base to 1024 B; at least 120 KB so that one CTA occupies an SM and
    // its 512-column TMEM allocation never waits for another CTA's
    static constexpr int kAlloc = (kBytes + 1024) > 120 * 1024 ? (kBytes + 1024) : 120 * 1024;
};

struct AttnParams {
    const __half* q;           // [B, H, S_q, D]
    float* out;                // [B, H, S_q, D]
    Buckets bk;
    const int32_t* rows;       // [H, S_kv] slot values of the stored entries, grouped by precision
    const int32_t* counts;     // [H, 5]: stored entries per precision, evicted entries
    int B, H, S_q, S_kv, G;
    float scale_log2;          // softmax scale * log2(e)
    int* err;
};

__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ uint32_t half2_bits(__half2 h) {
    uint32_t u;
    memcpy(&u, &h, 4);
    return u;
}

// Warp-uniform bounded wait: every lane polls, and the warp fails together if any lane gave
// up, so .sync.aligned tcgen05 instructions that follow stay convergent.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, int* err, int code) {
    const bool ok = mbar_wait(bar, parity, err, code);
    return __all_sync(0xffffffffu, ok);
}

__device__ __forceinline__ __half2 bits_half2(uint32_t u) {
    __half2 h;
    memcpy(&h, &u, 4);
    return h;
}

// Eight int8 codes (two words) -> eight exact fp16 values: (0x64 << 8 | (q ^ 0x80)) is
// 1024 + q + 128 in fp16, minus 1152.
__device__ __forceinline__ uint4 int8x8_to_half(uint32_t w0, uint32_t w1) {
    const __half2 bias = bits_half2(0x64806480u);
    const uint32_t x0 = w0 ^ 0x80808080u, x1 = w1 ^ 0x80808080u;
    uint4 r;
    r.x = half2_bits(__hsub2(bits_half2(__byte_perm(x0, 0x64646464u, 0x4140)), bias));
    r.y = half2_bits(__hsub2(bits_half2(__byte_perm(x0, 0x64646464u, 0x4342)), bias));
    r.z = half2_bits(__hsub2(bits_half2(__byte_perm(x1, 0x64646464u, 0x4140)), bias));
    r.w = half2_bits(__hsub2(bits_half2(__byte_perm(x1, 0x64646464u, 0x4342)), bias));
    return r;
}

// Eight int4 codes (one word, high nibble first per byte) times a group scale, computed in
// fp32 exactly as the reference dequantises ((nibble - 8) * scale), then rounded to fp16.
__device__ __forceinline__ uint4 int4x8_to_half(uint32_t w, float s) {
    float v[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint32_t byte = (w >> (8 * i)) & 0xFFu;
        v[2 * i] = __fmul_rn(__int_as_float(0x4B000000 | (byte >> 4)) - 8388616.0f, s);
        v[2 * i + 1] = __fmul_rn(__int_as_float(0x4B000000 | (byte & 0xF)) - 8388616.0f, s);
    }
    uint4 r;
    r.x = half2_bits(__floats2half2_rn(v[0], v[1]));
    r.y = half2_bits(__floats2half2_rn(v[2], v[3]));
    r.z = half2_bits(__floats2half2_rn(v[4], v[5]));
    r.w = half2_bits(__floats2half2_rn(v[6], v[7]));
    return r;
}

__device__ __forceinline__ uint4 f32x8_to_half(const float* p) {
    const float4 a = *reinterpret_cast<const float4*>(p);
    const float4 b = *reinterpret_cast<const float4*>(p + 4);
    uint4 r;
    r.x = half2_bits(__floats2half2_rn(a.x, a.y));
    r.y = half2_bits(__floats2half2_rn(a.z, a.w));
    r.z = half2_bits(__floats2half2_rn(b.x, b.y));
    r.w = half2_bits(__floats2half2_rn(b.z, b.w));
    return r;
}

// Raw packed bytes of one lane's share of one K row and one V row: chunk `l8` (8 values)
// of each 64-value atom, plus the row/group scales.  Loaded for several rows before any is
// converted, so a converter lane keeps several L2 requests in flight.
template <int NA>
struct RawRow {
    uint4 k[NA][2], v[NA][2];   // fp32 uses both halves, fp16 one, int8 8 bytes, int4 4 bytes
    float sk[NA], sv[NA];
    int code;                   // 0..3, or -1 for a padding row
};

template <int D>
__device__ __forceinline__ void load_raw_row(const AttnParams& p, int b, int32_t e, int l8, RawRow<D / 64>& r) {
    constexpr int NA = D / 64;
    r.code = e < 0 ? -1 : slot_code(e);
    if (e < 0) return;
    const int64_t row = (int64_t)slot_pos(e) * p.B + b;
    const skv_bucket& bb = p.bk.b[r.code];
#pragma unroll
    for (int a = 0; a < NA; ++a) {
        const int d0 = a * 64 + l8 * 8;
        if (r.code == 0) {
            const uint4* pk = reinterpret_cast<const uint4*>(reinterpret_cast<const float*>(bb.k) + row * D + d0);
            const uint4* pv = reinterpret_cast<const uint4*>(reinterpret_cast<const float*>(bb.v) + row * D + d0);
            r.k[a][0] = pk[0];
            r.k[a][1] = pk[1];
            r.v[a][0] = pv[0];
            r.v[a][1] = pv[1];
        } else if (r.code == 1) {
            r.k[a][0] = *reinterpret_cast<const uint4*>(reinterpret_cast<const __half*>(bb.k) + row * D + d0);
            r.v[a][0] = *reinterpret_cast<const uint4*>(reinterpret_cast<const __half*>(bb.v) + row * D + d0);
        } else if (r.code == 2) {
            const uint2 wk = *reinterpret_cast<const uint2*>(reinterpret_cast<const int8_t*>(bb.k) + row * D + d0);
            const uint2 wv = *reinterpret_cast<const uint2*>(reinterpret_cast<const int8_t*>(bb.v) + row * D + d0);
            r.k[a][0] = make_uint4(wk.x, wk.y, 0, 0);
            r.v[a][0] = make_uint4(wv.x, wv.y, 0, 0);
            if (a == 0) {
                r.sk[0] = bb.scale_k[row];
                r.sv[0] = bb.scale_v[row];
            }
        } else {
            const int64_t off = (int64_t)slot_pos(e) * ((int64_t)p.B * D / 2) + (int64_t)b * (D / 2) + d0 / 2;
            r.k[a][0].x = *reinterpret_cast<const uint32_t*>(reinterpret_cast<const uint8_t*>(bb.k) + off);
            r.v[a][0].x = *reinterpret_cast<const uint32_t*>(reinterpret_cast<const uint8_t*>(bb.v) + off);
            const int NG = D / p.G;
            const int g = d0 / p.G;
            r.sk[a] = bb.scale_k[row * NG + g];
            r.sv[a] = bb.scale_v[row * NG + g];
        }
    }
}

// Eight int8 codes times the row scale, in fp32 exactly as the reference dequantises
// (q * scale), then rounded to fp16.  (q ^ 0x80) | 0x4B000000 is 2^23 + q + 128.
__device__ __forceinline__ uint4 int8x8_scaled_to_half(uint32_t w0, uint32_t w1, float s) {
    float v[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        v[i] = __fmul_rn(__int_as_float(0x4B000000 | (((w0 >> (8 * i)) & 0xFFu) ^ 0x80u)) - 8388736.0f, s);
        v[4 + i] = __fmul_rn(__int_as_float(0x4B000000 | (((w1 >> (8 * i)) & 0xFFu) ^ 0x80u)) - 8388736.0f, s);
    }
    uint4 r;
    r.x = half2_bits(__floats2half2_rn(v[0], v[1]));
    r.y = half2_bits(__floats2half2_rn(v[2], v[3]));
    r.z = half2_bits(__floats2half2_rn(v[4], v[5]));
    r.w = half2_bits(__floats2half2_rn(v[6], v[7]));
    return r;
}

__device__ __forceinline__ uint4 f32x8_bits_to_half(const uint4& a, const uint4& b) {
    uint4 r;
    r.x = half2_bits(__floats2half2_rn(__uint_as_float(a.x), __uint_as_float(a.y)));
    r.y = half2_bits(__floats2half2_rn(__uint_as_float(a.z), __uint_as_float(a.w)));
    r.z = half2_bits(__floats2half2_rn(__uint_as_float(b.x), __uint_as_float(b.y)));
    r.w = half2_bits(__floats2half2_rn(__uint_as_float(b.z), __uint_as_float(b.w)));
    return r;
}

// Converts one lane's share of a K and a V row to fp16 and stores it, 128B-swizzled, at row
// `r` of the tiles (zeros for a padding row).
template <int D>
__device__ __forceinline__ void store_row(const RawRow<D / 64>& raw, int r, int l8, uint8_t* ktile, uint8_t* vtile) {
    constexpr int NA = D / 64;
#pragma unroll
    for (int a = 0; a < NA; ++a) {
        uint4 hk = make_uint4(0, 0, 0, 0), hv = make_uint4(0, 0, 0, 0);
        if (raw.code == 0) {
            hk = f32x8_bits_to_half(raw.k[a][0], raw.k[a][1]);
            hv = f32x8_bits_to_half(raw.v[a][0], raw.v[a][1]);
        } else if (raw.code == 1) {
            hk = raw.k[a][0];
            hv = raw.v[a][0];
        } else if (raw.code == 2) {
            hk = int8x8_scaled_to_half(raw.k[a][0].x, raw.k[a][0].y, raw.sk[0]);
            hv = int8x8_scaled_to_half(raw.v[a][0].x, raw.v[a][0].y, raw.sv[0]);
        } else if (raw.code == 3) {
            hk = int4x8_to_half(raw.k[a][0].x, raw.sk[a]);
            hv = int4x8_to_half(raw.v[a][0].x, raw.sv[a]);
        }
        *reinterpret_cast<uint4*>(ktile + a * kBN * 128 + sw128_offset(r, l8)) = hk;
        *reinterpret_cast<uint4*>(vtile + a * kBN * 128 + sw128_offset(r, l8)) = hv;
    }
}

__device__ __forceinline__ void converters_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kConvWarps * 32) : "memory"); }

template <int D>
__global__ void __launch_bounds__(kAttnThreads, 1) packed_attention_kernel(AttnParams p) {
    using L = AttnLayout<D>;
    constexpr int NA = L::NA;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int h = blockIdx.y, b = blockIdx.z;
    const int q0 = blockIdx.x * kBM;
    const int* cnt = p.counts + (int64_t)h * 5;
    const int n_stored = cnt[0] + cnt[1] + cnt[2] + cnt[3];
    const int n_ev = cnt[4];
    const int nt = (n_stored + kBN - 1) / kBN;

    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBar);
    uint64_t* kv_full = bars;                   // [kStages], count kConvWarps
    uint64_t* kv_empty = bars + kStages;        // [kStages], count 1 (commit)
    uint64_t* s_full = bars + 2 * kStages;      // [2], count 1 (commit)
    uint64_t* p_full = bars + 2 * kStages + 2;  // count kSoftmaxWarps
    uint64_t* pv_done = p_full + 1;             // count 1 (commit)
    uint64_t* mma_done = pv_done + 1;           // count 1 (commit), drain before TMEM release
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kTmemSlot);
    int32_t* ent = reinterpret_cast<int32_t*>(smem + L::kEnt);

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&kv_full[s], kConvWarps);
            mbar_init(&kv_empty[s], 1);
        }
        mbar_init(&s_full[0], 1);
        mbar_init(&s_full[1], 1);
        mbar_init(p_full, kSoftmaxWarps);
        mbar_init(pv_done, 1);
        mbar_init(mma_done, 1);
        fence_mbarrier_init();
    }
    constexpr int kMmaWarp = kSoftmaxWarps + kConvWarps;
    if (warp == kMmaWarp) {
        tmem_alloc(tmem_slot, kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t tS0 = tmem, tS1 = tmem + 128, tO = tmem + 256;

    if (warp < kSoftmaxWarps) {
        // ------------------------------------------------------------------ softmax
        const int t = threadIdx.x;                       // query row in the tile == TMEM lane
        const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
        const float sl2 = p.scale_log2;
        float m_ref = n_ev > 0 ? 0.0f : -INFINITY;       // evicted rows: logit 0
        float l = (float)n_ev;
        bool ok = true;
        for (int j = 0; j < nt && ok; ++j) {
            const int sb = j & 1;
            const uint32_t tS = sb ? tS1 : tS0;
            const int n_valid = min(kBN, n_stored - j * kBN);
            if (!warp_wait(&s_full[sb], (j >> 1) & 1, p.err, kErrSFull)) { ok = false; break; }
            tc_fence_after();
            uint32_t r[32];
            // pass 1: row max of the raw scores (scale > 0; padding columns score exactly 0,
            // which can only raise the reference max -- harmless)
            float mx0 = -INFINITY, mx1 = -INFINITY, mx2 = -INFINITY, mx3 = -INFINITY;
#pragma unroll
            for (int c = 0; c < kBN / 32; c += 2) {
                uint32_t r2[32];
                tmem_ld32(tS + lane_off + c * 32, r);
                tmem_ld32(tS + lane_off + (c + 1) * 32, r2);
                tmem_wait_ld();
#pragma unroll
                for (int i = 0; i < 32; i += 2) {
                    mx0 = fmaxf(mx0, __uint_as_float(r[i]));
                    mx1 = fmaxf(mx1, __uint_as_float(r[i + 1]));
                    mx2 = fmaxf(mx2, __uint_as_float(r2[i]));
                    mx3 = fmaxf(mx3, __uint_as_float(r2[i + 1]));
                }
            }
            const float mt = fmaxf(fmaxf(mx0, mx1), fmaxf(mx2, mx3)) * sl2;
            bool pv_seen = false;
            const bool need = mt > m_ref + kRescaleThreshold;
            if (__any_sync(0xffffffffu, need)) {
                // rows that keep their reference max use factor 1 (TMEM access is warp-wide)
                const float f = need ? ex2(m_ref - mt) : 1.0f;   // 0 when m_ref = -inf
                l *= f;
                if (j > 0) {
                    if (!warp_wait(pv_done, (j - 1) & 1, p.err, kErrPvDone)) { ok = false; break; }
                    pv_seen = true;
                    tc_fence_after();
#pragma unroll
                    for (int c = 0; c < D / 32; ++c) {
                        tmem_ld32(tO + lane_off + c * 32, r);
                        tmem_wait_ld();
#pragma unroll
                        for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * f);
                        tmem_st32(tO + lane_off + c * 32, r);
                    }
                    tmem_wait_st();
                }
                if (need) m_ref = mt;
            }
            if (j > 0 && !pv_seen) {
                // the single P buffer is still read by the previous tile's P*V
                if (!warp_wait(pv_done, (j - 1) & 1, p.err, kErrPvDone)) { ok = false; break; }
            }
            // pass 2: P = 2^(s*scale - m_ref) in fp16 into shared memory
            uint8_t* ptile = smem + L::kP;
            const float neg_m = -m_ref;
            float l0 = 0.f, l1 = 0.f, l2 = 0.f, l3 = 0.f;
#pragma unroll
            for (int c = 0; c < kBN / 32; ++c) {
                tmem_ld32(tS + lane_off + c * 32, r);
                tmem_wait_ld();
                float pv[32];
#pragma unroll
                for (int i = 0; i < 32; ++i) pv[i] = ex2(fmaf(__uint_as_float(r[i]), sl2, neg_m));
                if (n_valid < kBN) {
#pragma unroll
                    for (int i = 0; i < 32; ++i) pv[i] = (c * 32 + i < n_valid) ? pv[i] : 0.0f;
                }
                uint32_t hp[16];
#pragma unroll
                for (int i = 0; i < 32; i += 4) {
                    l0 += pv[i];
                    l1 += pv[i + 1];
                    l2 += pv[i + 2];
                    l3 += pv[i + 3];
                    hp[i / 2] = half2_bits(__floats2half2_rn(pv[i], pv[i + 1]));
                    hp[i / 2 + 1] = half2_bits(__floats2half2_rn(pv[i + 2], pv[i + 3]));
                }
                // columns c*32 .. c*32+31 = 4 chunks of 8 in atom c/2
                uint8_t* atom = ptile + (c >> 1) * kBM * 128;
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const int chunk = (c & 1) * 4 + k;
                    *reinterpret_cast<uint4*>(atom + sw128_offset(t, chunk)) =
                        make_uint4(hp[4 * k], hp[4 * k + 1], hp[4 * k + 2], hp[4 * k + 3]);
                }
            }
            l += (l0 + l1) + (l2 + l3);
            tc_fence_before();
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(p_full);
        }
        // epilogue: O / l
        const bool row_ok = q0 + t < p.S_q;
        float* orow = p.out + (((int64_t)b * p.H + h) * p.S_q + (q0 + t)) * D;
        ok = __all_sync(0xffffffffu, ok);
        if (nt == 0 || !ok) {
            if (row_ok)
                for (int d = 0; d < D; d += 4) *reinterpret_cast<float4*>(orow + d) = make_float4(0.f, 0.f, 0.f, 0.f);
        } else {
            const bool done = warp_wait(pv_done, (nt - 1) & 1, p.err, kErrPvDone);
            tc_fence_after();
            const float inv = (done && l > 0.0f) ? 1.0f / l : 0.0f;
            uint32_t r[32];
#pragma unroll
            for (int c = 0; c < D / 32; ++c) {
                tmem_ld32(tO + lane_off + c * 32, r);
                tmem_wait_ld();
                if (row_ok) {
#pragma unroll
                    for (int i = 0; i < 32; i += 4)
                        *reinterpret_cast<float4*>(orow + c * 32 + i) =
                            make_float4(__uint_as_float(r[i]) * inv, __uint_as_float(r[i + 1]) * inv,
                                        __uint_as_float(r[i + 2]) * inv, __uint_as_float(r[i + 3]) * inv);
                }
            }
        }
    } else if (warp < kSoftmaxWarps + kConvWarps) {
        // --------------------------------------------------------------- converters
        const int wc = warp - kSoftmaxWarps;
        const int ctid = threadIdx.x - kSoftmaxWarps * 32;      // 0 .. 32*kConvWarps-1
        const int lrow = lane >> 3, l8 = lane & 7;
        uint8_t* qtile = smem + L::kQ;
        const int32_t* hrows = p.rows + (int64_t)h * p.S_kv;
        int32_t next_e = (ctid < kBN && ctid < n_stored) ? hrows[ctid] : -1;   // entry list of tile 0
        constexpr int kRowsPerStep = kConvWarps * 4;
        for (int step = 0; step < kBM / kRowsPerStep; ++step) {
            const int r = step * kRowsPerStep + wc * 4 + lrow;
            const int qi = q0 + r;
#pragma unroll
            for (int a = 0; a < NA; ++a) {
                uint4 v = make_uint4(0, 0, 0, 0);
                if (qi < p.S_q)
                    v = *reinterpret_cast<const uint4*>(p.q + (((int64_t)b * p.H + h) * p.S_q + qi) * D + a * 64 + l8 * 8);
                *reinterpret_cast<uint4*>(qtile + a * kBM * 128 + sw128_offset(r, l8)) = v;
            }
        }
        constexpr int kRowsPerBatch = 2;       // rows whose loads are in flight together
        volatile int* conv_fail = reinterpret_cast<volatile int*>(smem + L::kTmemSlot + 8);
        if (ctid == 0) *conv_fail = 0;
        converters_sync();
        for (int j = 0; j < nt; ++j) {
            const int s = j % kStages;
            const bool ok = j < kStages || warp_wait(&kv_empty[s], ((j / kStages) - 1) & 1, p.err, kErrKvEmpty);
            if (!ok && lane == 0) *conv_fail = 1;
            int32_t* e_tile = ent + s * kBN;
            if (ok && ctid < kBN) e_tile[ctid] = next_e;
            const int nxt = (j + 1) * kBN + ctid;
            next_e = (ctid < kBN && j + 1 < nt && nxt < n_stored) ? hrows[nxt] : -1;
            // every converter warp reaches this barrier on every tile, so one warp's timeout
            // stops all four together instead of leaving the others waiting here
            converters_sync();
            if (*conv_fail) break;
            uint8_t* ktile = smem + L::kK + s * NA * kBN * 128;
            uint8_t* vtile = smem + L::kV + s * NA * kBN * 128;
            for (int step = 0; step < kBN / kRowsPerStep; step += kRowsPerBatch) {
                RawRow<NA> raw[kRowsPerBatch];
#pragma unroll
                for (int i = 0; i < kRowsPerBatch; ++i) {
                    const int r = (step + i) * kRowsPerStep + wc * 4 + lrow;
                    load_raw_row<D>(p, b, e_tile[r], l8, raw[i]);
                }
#pragma unroll
                for (int i = 0; i < kRowsPerBatch; ++i) {
                    const int r = (step + i) * kRowsPerStep + wc * 4 + lrow;
                    store_row<D>(raw[i], r, l8, ktile, vtile);
                }
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(&kv_full[s]);
        }
    } else {
        // ----------------------------------------------------------------- MMA issue
        if (lane == 0 && nt > 0) {
            const uint32_t idesc_s = idesc_f16_f32(kBM, kBN, false, false);
            const uint32_t idesc_o = idesc_f16_f32(kBM, D, false, true);
            const uint32_t q_base = smem_u32(smem + L::kQ);
            const uint32_t p_base = smem_u32(smem + L::kP);
            bool ok = true;
            auto issue_pv = [&](int i) -> bool {
                if (!mbar_wait(p_full, i & 1, p.err, kErrPFull)) return false;
                tc_fence_after();
                const uint32_t v_base = smem_u32(smem + L::kV + (i % kStages) * NA * kBN * 128);
#pragma unroll
                for (int k = 0; k < kBN / 16; ++k) {
                    const uint64_t adesc = smem_desc_sw128(p_base + (k >> 2) * kBM * 128 + (k & 3) * 32, 16, 1024);
                    const uint64_t bdesc = smem_desc_sw128(v_base + k * 16 * 128, kBN * 128, 1024);
                    umma_f16(tO, adesc, bdesc, idesc_o, (i > 0 || k > 0) ? 1u : 0u);
                }
                umma_commit(pv_done);
                umma_commit(&kv_empty[i % kStages]);
                return true;
            };
            for (int j = 0; j < nt && ok; ++j) {
                const int s = j % kStages, sb = j & 1;
                if (!mbar_wait(&kv_full[s], (j / kStages) & 1, p.err, kErrKvFull)) { ok = false; break; }
                tc_fence_after();
                const uint32_t k_base = smem_u32(smem + L::kK + s * NA * kBN * 128);
#pragma unroll
                for (int k = 0; k < D / 16; ++k) {
                    const uint32_t off = (k >> 2) * kBM * 128 + (k & 3) * 32;
                    const uint32_t koff = (k >> 2) * kBN * 128 + (k & 3) * 32;
                    const uint64_t adesc = smem_desc_sw128(q_base + off, 16, 1024);
                    const uint64_t bdesc = smem_desc_sw128(k_base + koff, 16, 1024);
                    umma_f16(sb ? tS1 : tS0, adesc, bdesc, idesc_s, k > 0 ? 1u : 0u);
                }
                umma_commit(&s_full[sb]);
                if (j > 0 && !issue_pv(j - 1)) { ok = false; break; }
            }
            if (ok) issue_pv(nt - 1);
            // drain: every UMMA issued above completes before TMEM is released
            umma_commit(mma_done);
            mbar_wait(mma_done, 0, p.err, kErrDrain);
        }
        __syncwarp();
    }

    tc_fence_before();
    __syncthreads();
    if (warp == kMmaWarp) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

// ---------------------------------------------------------------------------------------
// per-head row index
// ---------------------------------------------------------------------------------------
constexpr int kHiThreads = 1024;

__global__ void __launch_bounds__(kHiThreads) head_index_kernel(const int32_t* __restrict__ slot, int S, int H,
                                                                int32_t* __restrict__ rows, int32_t* __restrict__ counts) {
    const int h = blockIdx.x;
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    __shared__ int s_red[5][32];
    __shared__ int s_base[4];
    __shared__ int s_warp[4][32];
    int c0 = 0, c1 = 0, c2 = 0, c3 = 0, c4 = 0;
    for (int t = threadIdx.x; t < S; t += kHiThreads) {
        const int32_t sl = slot[(int64_t)t * H + h];
        const int code = sl < 0 ? 4 : slot_code(sl);
        c0 += code == 0;
        c1 += code == 1;
        c2 += code == 2;
        c3 += code == 3;
        c4 += code == 4;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        c0 += __shfl_xor_sync(0xffffffffu, c0, o);
        c1 += __shfl_xor_sync(0xffffffffu, c1, o);
        c2 += __shfl_xor_sync(0xffffffffu, c2, o);
        c3 += __shfl_xor_sync(0xffffffffu, c3, o);
        c4 += __shfl_xor_sync(0xffffffffu, c4, o);
    }
    if (lane == 0) {
        s_red[0][w] = c0;
        s_red[1][w] = c1;
        s_red[2][w] = c2;
        s_red[3][w] = c3;
        s_red[4][w] = c4;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int base = 0;
        for (int k = 0; k < 5; ++k) {
            int v = 0;
            for (int q = 0; q < kHiThreads / 32; ++q) v += s_red[k][q];
            if (k < 4) s_base[k] = base;
            base += v;
            counts[(int64_t)h * 5 + k] = v;
        }
    }
    __syncthreads();
    int r0 = s_base[0], r1 = s_base[1], r2 = s_base[2], r3 = s_base[3];
    for (int t0 = 0; t0 < S; t0 += kHiThreads) {
        const int t = t0 + threadIdx.x;
        const int32_t sl = t < S ? slot[(int64_t)t * H + h] : -1;
        const int code = sl < 0 ? 4 : slot_code(sl);
        const unsigned m0 = __ballot_sync(0xffffffffu, code == 0);
        const unsigned m1 = __ballot_sync(0xffffffffu, code == 1);
        const unsigned m2 = __ballot_sync(0xffffffffu, code == 2);
        const unsigned m3 = __ballot_sync(0xffffffffu, code == 3);
        if (lane == 0) {
            s_warp[0][w] = __popc(m0);
            s_warp[1][w] = __popc(m1);
            s_warp[2][w] = __popc(m2);
            s_warp[3][w] = __popc(m3);
        }
        __syncthreads();
        if (code < 4) {
            const unsigned m = code == 0 ? m0 : (code == 1 ? m1 : (code == 2 ? m2 : m3));
            const int run = code == 0 ? r0 : (code == 1 ? r1 : (code == 2 ? r2 : r3));
            int before = 0;
            for (int q = 0; q < w; ++q) before += s_warp[code][q];
            rows[(int64_t)h * S + run + before + __popc(m & ((1u << lane) - 1u))] = sl;
        }
        int t0s = 0, t1s = 0, t2s = 0, t3s = 0;
        for (int q = 0; q < kHiThreads / 32; ++q) {
            t0s += s_warp[0][q];
            t1s += s_warp[1][q];
            t2s += s_warp[2][q];
            t3s += s_warp[3][q];
        }
        r0 += t0s;
        r1 += t1s;
        r2 += t2s;
        r3 += t3s;
        __syncthreads();
    }
}

}  // namespace skv

using namespace skv;

extern "C" {

int skv_head_index(const int32_t* slot, int S, int H, int32_t* rows, int32_t* counts, void* stream) {
    if (!slot || !rows || !counts) return fail(SKV_ERR_INVALID_ARGUMENT, "head_index: null pointer");
    if (S <= 0 || H <= 0) return fail(SKV_ERR_INVALID_ARGUMENT, "head_index: bad shape");
    head_index_kernel<<<H, kHiThreads, 0, as_stream(stream)>>>(slot, S, H, rows, counts);
    return check_launch("head_index");
}

int skv_packed_attention(const void* q, int B, int H, int S_q, int D, const skv_bucket* buckets, int S_kv,
                         int int4_group, const int32_t* rows, const int32_t* counts, float scale, float* out,
                         int32_t* error_flag, void* stream) {
    if (!q || !buckets || !rows || !counts || !out || !error_flag)
        return fail(SKV_ERR_INVALID_ARGUMENT, "packed_attention: null pointer");
    if (B <= 0 || H <= 0 || S_q <= 0 || S_kv <= 0) return fail(SKV_ERR_INVALID_ARGUMENT, "packed_attention: bad shape");
    if (D != 64 && D != 128) return fail(SKV_ERR_UNSUPPORTED, "packed_attention: head_dim %d (64 or 128 supported)", D);
    const int G = int4_group > 0 && D % int4_group == 0 ? int4_group : D;
    if (G % 8) return fail(SKV_ERR_UNSUPPORTED, "packed_attention: int4 group %d must be a multiple of 8", G);
    for (int p = 0; p < kNumBuckets; ++p) {
        if (buckets[p].count == 0) continue;
        const uintptr_t a = reinterpret_cast<uintptr_t>(buckets[p].k) | reinterpret_cast<uintptr_t>(buckets[p].v);
        if (a & 15) return fail(SKV_ERR_UNSUPPORTED, "packed_attention: bucket %d not 16-byte aligned", p);
    }
    if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(out)) & 15)
        return fail(SKV_ERR_UNSUPPORTED, "packed_attention: q/out not 16-byte aligned");
    AttnParams prm;
    prm.q = reinterpret_cast<const __half*>(q);
    prm.out = out;
    for (int p = 0; p < kNumBuckets; ++p) prm.bk.b[p] = buckets[p];
    prm.rows = rows;
    prm.counts = counts;
    prm.B = B;
    prm.H = H;
    prm.S_q = S_q;
    prm.S_kv = S_kv;
    prm.G = G;
    prm.scale_log2 = scale * 1.4426950408889634f;
    prm.err = error_flag;
    cudaStream_t s = as_stream(stream);
    if (cudaMemsetAsync(error_flag, 0, sizeof(int32_t), s) != cudaSuccess)
        return fail(SKV_ERR_CUDA, "packed_attention: memset failed");
    const dim3 grid((unsigned)((S_q + kBM - 1) / kBM), (unsigned)H, (unsigned)B);
    if (D == 128) {
        const int smem = AttnLayout<128>::kAlloc;
        cudaFuncSetAttribute(packed_attention_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        packed_attention_kernel<128><<<grid, kAttnThreads, smem, s>>>(prm);
    } else {
        const int smem = AttnLayout<64>::kAlloc;
        cudaFuncSetAttribute(packed_attention_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        packed_attention_kernel<64><<<grid, kAttnThreads, smem, s>>>(prm);
    }
    return check_launch("packed_attention");
}

}  // extern "C"
