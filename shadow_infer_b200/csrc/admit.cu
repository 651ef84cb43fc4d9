// KV sensitivity and budget admission.
//
//  * skv_kv_sensitivity -- kv_sensitivity (shadowinfer/shadowkv/rd_allocator.py:47-61):
//    (amax|k|^2 + amax|v|^2)/2 over batch and head_dim, one warp per (h, t), written [S,H].
//  * skv_admit_codes    -- admit_codes (rd_allocator.py:190-318).  The reference sorts all
//    (t,h) by score = importance*sensitivity (stable) and walks prefix sums of the downgrade
//    ladder.  Only the crossing point of those prefix sums matters, so this is done as a
//    WEIGHTED RADIX SELECT instead of a sort: every candidate gets a unique 64-bit key
//    (order-preserving score bits << 32 | flat index, which reproduces the stable tie
//    order), and 8-bit digit passes histogram the candidate weights (ladder savings for the
//    downgrade phase, entry costs for the eviction phase) until the unique boundary entry
//    is found.  All passes run in one cooperative launch: blocks meet at a bounded grid
//    barrier after each pass, every block scans the same 256-bin histogram and narrows the
//    key prefix identically, and a final sweep writes the new codes, the predicted bytes
//    and the eviction count.
#include <math.h>

#include "skv_common.cuh"

namespace skv {

// ---------------------------------------------------------------------------------------
// sensitivity
// ---------------------------------------------------------------------------------------
// Generic shapes: one warp per (h, t), lanes strided over D.
__global__ void __launch_bounds__(256) sensitivity_kernel(const float* __restrict__ k,
                                                          const float* __restrict__ v, int B, int H,
                                                          int S, int D, float* __restrict__ sens) {
    const int lane = threadIdx.x & 31;
    const int64_t n = (int64_t)H * S;
    const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    for (int64_t r = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < n; r += nwarps) {
        const int64_t h = r / S, t = r - h * S;
        float mk = 0.0f, mv = 0.0f;
        for (int b = 0; b < B; ++b) {
            const int64_t off = (((int64_t)b * H + h) * S + t) * D;
            for (int i = lane; i < D; i += 32) {
                mk = fmaxf(mk, fabsf(k[off + i]));
                mv = fmaxf(mv, fabsf(v[off + i]));
            }
        }
        mk = warp_max(mk);
        mv = warp_max(mv);
        if (lane == 0) sens[t * H + h] = __fdiv_rn(__fadd_rn(__fmul_rn(mk, mk), __fmul_rn(mv, mv)), 2.0f);
    }
}

// D == 128: grid x over token chunks (8 warps * RPW rows), y over heads; each warp keeps
// 2*RPW 128-bit loads in flight per batch.
template <int RPW>
__global__ void __launch_bounds__(256) sensitivity_d128_kernel(const float* __restrict__ k,
                                                               const float* __restrict__ v, int B, int H,
                                                               int S, float* __restrict__ sens) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int h = blockIdx.y;
    const int t0 = (blockIdx.x * 8 + warp) * RPW;
    if (t0 >= S) return;
    float mk[RPW], mv[RPW];
#pragma unroll
    for (int i = 0; i < RPW; ++i) mk[i] = mv[i] = 0.0f;
    for (int b = 0; b < B; ++b) {
        const int64_t base = (((int64_t)b * H + h) * S) * 128 + lane * 4;
        float4 a[RPW], c[RPW];
#pragma unroll
        for (int i = 0; i < RPW; ++i) {
            if (t0 + i < S) {
                a[i] = __ldcs(reinterpret_cast<const float4*>(k + base + (int64_t)(t0 + i) * 128));
                c[i] = __ldcs(reinterpret_cast<const float4*>(v + base + (int64_t)(t0 + i) * 128));
            } else {
                a[i] = c[i] = make_float4(0.f, 0.f, 0.f, 0.f);
            }
        }
#pragma unroll
        for (int i = 0; i < RPW; ++i) {
            mk[i] = fmaxf(mk[i], fmaxf(fmaxf(fabsf(a[i].x), fabsf(a[i].y)), fmaxf(fabsf(a[i].z), fabsf(a[i].w))));
            mv[i] = fmaxf(mv[i], fmaxf(fmaxf(fabsf(c[i].x), fabsf(c[i].y)), fmaxf(fabsf(c[i].z), fabsf(c[i].w))));
        }
    }
#pragma unroll
    for (int i = 0; i < RPW; ++i) {
        const float a = warp_max(mk[i]);
        const float c = warp_max(mv[i]);
        if (lane == i && t0 + i < S)
            sens[(int64_t)(t0 + i) * H + h] = __fdiv_rn(__fadd_rn(__fmul_rn(a, a), __fmul_rn(c, c)), 2.0f);
    }
}

// ---------------------------------------------------------------------------------------
// admission
// ---------------------------------------------------------------------------------------
struct AdmitHeader {
    long long predicted0;
    long long predicted_a;
    long long predicted_final;
    long long evicted;
    long long rem;                 // weight still to cover inside the current key prefix
    long long total;               // unused slot kept for layout stability
    unsigned long long prefix;     // key bits decided so far
    unsigned long long pmask;      // which bits are decided
    unsigned long long a_key;      // boundary key of the downgrade phase
    unsigned long long b_key;      // boundary key of the eviction phase
    int a_active, a_notenough, a_done, a_newcode;
    int b_active, b_notenough, b_done, pad0;
    unsigned int counter;          // last-block ticket
    unsigned int pad1;
};

struct AdmitArgs {
    const int8_t* codes;
    const float* imp;
    const float* sens;       // nullable -> ones
    const uint8_t* prot;     // nullable
    int8_t* out;
    long long* result;
    int64_t n;
    int H;
    int sink;
    int rd;
    int allow_evict;
    long long budget;
    long long cost[5];
    long long wA[5];         // total ladder savings of a base code (step1+step2+step3)
    long long delta[3];      // cost[c] - cost[c+1], c = 0..2
};

__device__ __forceinline__ uint32_t score_bits(float f) {
    if (f != f) return 0xFFFFFFFFu;       // NaN sorts last
    if (f == 0.0f) f = 0.0f;              // -0.0 ties with +0.0
    const uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__device__ __forceinline__ bool eligible(const AdmitArgs& a, int64_t i) {
    if (i / a.H < a.sink) return false;
    if (a.prot && a.prot[i]) return false;
    return true;
}

__device__ __forceinline__ unsigned long long entry_key(const AdmitArgs& a, int64_t i) {
    const float imp = a.imp[i];
    const float s = (a.rd && a.sens) ? __fmul_rn(imp, a.sens[i]) : imp;
    return ((unsigned long long)score_bits(s) << 32) | (unsigned long long)i;
}

__device__ __forceinline__ int code_after_a(const AdmitHeader& st, int base, unsigned long long key) {
    if (!st.a_active || base < 0 || base > 4) return base;
    if (st.a_notenough || key < st.a_key) return base != 4 ? 3 : 4;
    if (key == st.a_key) return st.a_newcode;
    return base;
}

__device__ __forceinline__ long long cost_of(const AdmitArgs& a, int code) {
    return (code >= 0 && code <= 4) ? a.cost[code] : 0;
}

// ---------------------------------------------------------------------------------------
// Persistent admission: every phase and digit pass of the radix select in ONE cooperative
// launch.  Blocks meet at a bounded grid barrier after each histogram pass; each pass has its
// own global histogram (no zeroing between passes), and every block derives the same
// selection state from it, so no block has to broadcast decisions.
// ---------------------------------------------------------------------------------------
constexpr int kAdmitMaxPasses = 8;                     // 4 score digits + up to 4 index digits

struct AdmitScratch {
    unsigned long long hist[2 * kAdmitMaxPasses][256];
    long long sums[4];                                 // predicted0, predicted_final, evicted, -
    unsigned bar_count, bar_gen;
    int err, pad;
};

struct AdmitPlanDigits {
    int shift[kAdmitMaxPasses];
    int n;
};

// Bounded grid barrier (cooperative launch guarantees every block is resident).  Returns
// false, and records the failure, if the other blocks do not arrive within the limit.
__device__ bool grid_barrier(AdmitScratch* sc, unsigned nblocks) {
    __shared__ int s_ok;
    __syncthreads();
    if (threadIdx.x == 0) {
        volatile unsigned* gen = &sc->bar_gen;
        const unsigned g = *gen;
        __threadfence();
        int ok = 1;
        if (atomicAdd(&sc->bar_count, 1u) == nblocks - 1) {
            sc->bar_count = 0;
            __threadfence();
            atomicAdd(&sc->bar_gen, 1u);
        } else {
            long long it = 0;
            while (*gen == g) {
                if (++it > (1ll << 24) || *reinterpret_cast<volatile int*>(&sc->err)) {
                    atomicExch(&sc->err, 1);
                    ok = 0;
                    break;
                }
                __nanosleep(32);
            }
        }
        __threadfence();
        s_ok = ok;
    }
    __syncthreads();
    return s_ok != 0;
}

__global__ void __launch_bounds__(256) admit_persistent_kernel(AdmitArgs a, AdmitScratch* sc, AdmitPlanDigits dg) {
    __shared__ unsigned long long s_hist[256];
    __shared__ long long s_inc[256];
    __shared__ long long s_red[8];
    __shared__ AdmitHeader st;                         // identical in every block
    __shared__ int s_found;
    const unsigned nblocks = gridDim.x;
    const int tid = threadIdx.x;
    bool ok = true;

    // predicted bytes of the input codes
    long long acc = 0;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + tid; i < a.n; i += (int64_t)nblocks * blockDim.x)
        acc += cost_of(a, a.codes[i]);
    acc = warp_sum_ll(acc);
    if ((tid & 31) == 0) s_red[tid >> 5] = acc;
    __syncthreads();
    if (tid == 0) {
        long long t = 0;
        for (int k = 0; k < 8; ++k) t += s_red[k];
        if (t) atomicAdd((unsigned long long*)&sc->sums[0], (unsigned long long)t);
    }
    ok = grid_barrier(sc, nblocks);
    if (tid == 0) {
        const long long p0 = (long long)__ldcg((const unsigned long long*)&sc->sums[0]);
        memset(&st, 0, sizeof(st));
        st.predicted0 = p0;
        st.predicted_a = p0;
        st.a_active = (a.budget >= 0 && p0 > a.budget) ? 1 : 0;
        st.rem = p0 - a.budget;
    }
    __syncthreads();

    int hist_id = 0;
    for (int phase = 0; phase < 2 && ok; ++phase) {
        if (phase == 0 && !st.a_active) continue;
        if (phase == 1 && !st.b_active) break;
        for (int pass = 0; pass < dg.n && ok; ++pass, ++hist_id) {
            if (phase == 0 ? st.a_done : st.b_done) break;
            const int shift = dg.shift[pass];
            s_hist[tid] = 0;
            __syncthreads();
            const unsigned long long prefix = st.prefix, pmask = st.pmask;
            for (int64_t i = blockIdx.x * (int64_t)blockDim.x + tid; i < a.n; i += (int64_t)nblocks * blockDim.x) {
                if (!eligible(a, i)) continue;
                const unsigned long long key = entry_key(a, i);
                if ((key & pmask) != prefix) continue;
                const int base = a.codes[i];
                const long long w = phase == 0 ? ((base >= 0 && base <= 4) ? a.wA[base] : 0)
                                               : cost_of(a, code_after_a(st, base, key));
                if (w) atomicAdd(&s_hist[(key >> shift) & 0xFF], (unsigned long long)w);
            }
            __syncthreads();
            if (s_hist[tid]) atomicAdd(&sc->hist[hist_id][tid], s_hist[tid]);
            ok = grid_barrier(sc, nblocks);
            if (!ok) break;
            // every block scans the same global histogram
            s_inc[tid] = (long long)__ldcg(&sc->hist[hist_id][tid]);
            if (tid == 0) s_found = 256;
            __syncthreads();
            for (int o = 1; o < 256; o <<= 1) {
                const long long add = tid >= o ? s_inc[tid - o] : 0;
                __syncthreads();
                s_inc[tid] += add;
                __syncthreads();
            }
            const long long rem = st.rem;
            if (s_inc[tid] >= rem) atomicMin(&s_found, tid);
            __syncthreads();
            if (tid == 0) {
                const int d = s_found;
                if (d == 256) {
                    // all candidate weight falls short: the whole candidate list is consumed
                    if (phase == 0) {
                        st.a_notenough = 1;
                        st.a_done = 1;
                        st.predicted_a = st.predicted0 - s_inc[255];
                    } else {
                        st.b_notenough = 1;
                        st.b_done = 1;
                    }
                } else {
                    const long long before = d > 0 ? s_inc[d - 1] : 0;
                    st.rem = rem - before;
                    st.prefix |= (unsigned long long)d << shift;
                    st.pmask |= 0xFFull << shift;
                    if (pass == dg.n - 1) {
                        const unsigned long long key = st.prefix;
                        if (phase == 0) {
                            const int64_t idx = (int64_t)(key & 0xFFFFFFFFull);
                            const int base = a.codes[idx];
                            const long long r = st.rem;
                            const long long s1 = base < 3 ? a.delta[base] : 0;
                            const int n1 = base < 3 ? base + 1 : base;
                            const long long s2 = n1 < 3 ? a.delta[n1] : 0;
                            const int n2 = n1 < 3 ? n1 + 1 : n1;
                            int nc = base;
                            if (base != 4) nc = r <= s1 ? n1 : (r <= s1 + s2 ? n2 : 3);
                            st.a_key = key;
                            st.a_newcode = nc;
                            st.a_done = 1;
                            const long long consumed = (st.predicted0 - a.budget) - r;
                            st.predicted_a = st.predicted0 - consumed - (a.cost[base] - a.cost[nc]);
                        } else {
                            st.b_key = key;
                            st.b_done = 1;
                        }
                    }
                }
                if (phase == 0 && st.a_done) {
                    st.b_active = (a.allow_evict && st.predicted_a > a.budget) ? 1 : 0;
                    st.rem = st.predicted_a - a.budget;
                    st.prefix = 0;
                    st.pmask = 0;
                }
            }
            __syncthreads();
        }
    }

    // apply: final codes, predicted bytes, evictions
    long long pred = 0, ev = 0;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + tid; i < a.n; i += (int64_t)nblocks * blockDim.x) {
        const int base = a.codes[i];
        int code = base;
        if (ok && eligible(a, i) && (st.a_active || st.b_active)) {
            const unsigned long long key = entry_key(a, i);
            code = code_after_a(st, base, key);
            if (st.b_active && (st.b_notenough || key <= st.b_key)) {
                if (code != 4) ++ev;
                code = 4;
            }
        }
        a.out[i] = (int8_t)code;
        pred += cost_of(a, code);
    }
    pred = warp_sum_ll(pred);
    ev = warp_sum_ll(ev);
    __shared__ long long s_e[8];
    if ((tid & 31) == 0) {
        s_red[tid >> 5] = pred;
        s_e[tid >> 5] = ev;
    }
    __syncthreads();
    if (tid == 0) {
        long long tp = 0, te = 0;
        for (int k = 0; k < 8; ++k) {
            tp += s_red[k];
            te += s_e[k];
        }
        if (tp) atomicAdd((unsigned long long*)&sc->sums[1], (unsigned long long)tp);
        if (te) atomicAdd((unsigned long long*)&sc->sums[2], (unsigned long long)te);
    }
    const bool fin = grid_barrier(sc, nblocks);
    if (blockIdx.x == 0 && tid == 0) {
        const bool good = ok && fin && __ldcg(&sc->err) == 0;
        a.result[0] = good ? (long long)__ldcg((const unsigned long long*)&sc->sums[1]) : -1;
        a.result[1] = good ? (long long)__ldcg((const unsigned long long*)&sc->sums[2]) : -1;
    }
}

static int admit_coop_blocks(int64_t n) {
    static int cached[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    int per_sm = 0;
    if (dev >= 0 && dev < 64 && cached[dev] > 0) {
        per_sm = cached[dev];
    } else {
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, admit_persistent_kernel, 256, 0) != cudaSuccess ||
            per_sm <= 0)
            per_sm = 1;
        if (dev >= 0 && dev < 64) cached[dev] = per_sm;
    }
    const int64_t cap = (int64_t)sm_count() * (per_sm < 2 ? per_sm : 2);
    const int64_t want = (n + 1023) / 1024;
    return (int)(want < 1 ? 1 : (want < cap ? want : cap));
}

static long long entry_cost(int code, int B, int D, int group_size) {
    const int g = (group_size > 0 && D % group_size == 0) ? group_size : D;
    switch (code) {
        case 0: return (long long)((double)B * D * 4 * 2.0);
        case 1: return (long long)((double)B * D * 2 * 2.0);
        case 2: return (long long)(((double)B * D + (double)B * 4) * 2.0);
        case 3: return (long long)(((double)B * D / 2.0 + (double)B * (D / g) * 4) * 2.0);
        default: return 0;
    }
}

}  // namespace skv

using namespace skv;

extern "C" {

int skv_kv_sensitivity(const float* k, const float* v, int B, int H, int S, int D, float* sensitivity,
                       void* stream) {
    if (!k || !v || !sensitivity) return fail(SKV_ERR_INVALID_ARGUMENT, "kv_sensitivity: null pointer");
    if (B <= 0 || H <= 0 || S <= 0 || D <= 0) return fail(SKV_ERR_INVALID_ARGUMENT, "kv_sensitivity: bad shape");
    if (D == 128 && ((reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v)) & 15) == 0) {
        constexpr int kRPW = 4;
        const dim3 grid((unsigned)((S + 8 * kRPW - 1) / (8 * kRPW)), (unsigned)H);
        sensitivity_d128_kernel<kRPW><<<grid, 256, 0, as_stream(stream)>>>(k, v, B, H, S, sensitivity);
        return check_launch("kv_sensitivity");
    }
    const int64_t n = (int64_t)H * S;
    const int64_t want = (n + 7) / 8;
    const int blocks = (int)(want < (int64_t)sm_count() * 8 ? want : (int64_t)sm_count() * 8);
    sensitivity_kernel<<<blocks, 256, 0, as_stream(stream)>>>(k, v, B, H, S, D, sensitivity);
    return check_launch("kv_sensitivity");
}

size_t skv_admit_scratch_bytes(int S, int H) {
    (void)S;
    (void)H;
    return sizeof(AdmitScratch);
}

int skv_admit_codes(const int8_t* codes_in, int8_t* codes_out, const float* importance, const float* sensitivity,
                    const uint8_t* protected_mask, int S, int H, int64_t budget_bytes, int batch, int head_dim,
                    int group_size, int sink_tokens, int rd_allocation, int allow_eviction, void* scratch,
                    size_t scratch_bytes, int64_t* result, void* stream) {
    if (S <= 0 || H <= 0) return fail(SKV_ERR_INVALID_ARGUMENT, "admit_codes: bad shape");
    if (!codes_in || !codes_out || !importance || !scratch || !result)
        return fail(SKV_ERR_INVALID_ARGUMENT, "admit_codes: null pointer");
    if (scratch_bytes < sizeof(AdmitScratch))
        return fail(SKV_ERR_SCRATCH, "admit_codes: scratch %zu < %zu", scratch_bytes, sizeof(AdmitScratch));
    const int64_t n = (int64_t)S * H;
    if (n > (int64_t(1) << 31)) return fail(SKV_ERR_TOO_LARGE, "admit_codes: S*H above 2^31");
    AdmitArgs a;
    a.codes = codes_in;
    a.imp = importance;
    a.sens = sensitivity;
    a.prot = protected_mask;
    a.out = codes_out;
    a.result = (long long*)result;
    a.n = n;
    a.H = H;
    a.sink = sink_tokens > 0 ? sink_tokens : 0;
    a.rd = rd_allocation;
    a.allow_evict = allow_eviction;
    a.budget = budget_bytes;
    for (int c = 0; c < 5; ++c) a.cost[c] = entry_cost(c, batch, head_dim, group_size);
    for (int c = 0; c < 3; ++c) a.delta[c] = a.cost[c] - a.cost[c + 1];
    for (int c = 0; c < 5; ++c) {
        long long w = 0;
        for (int x = c; x < 3; ++x) w += a.delta[x];
        a.wA[c] = c < 3 ? w : 0;
    }
    cudaStream_t s = as_stream(stream);
    AdmitScratch* sc = reinterpret_cast<AdmitScratch*>(scratch);
    if (cudaMemsetAsync(sc, 0, sizeof(AdmitScratch), s) != cudaSuccess)
        return fail(SKV_ERR_CUDA, "admit_codes: memset failed");
    // digit shifts: 4 score digits, then enough index digits to cover n-1
    int idx_bits = 0;
    while (idx_bits < 63 && ((int64_t)1 << idx_bits) < n) ++idx_bits;
    const int idx_digits = (idx_bits + 7) / 8;
    AdmitPlanDigits dg;
    dg.n = 0;
    for (int d = 3; d >= 0; --d) dg.shift[dg.n++] = 32 + 8 * d;
    for (int d = idx_digits - 1; d >= 0; --d) dg.shift[dg.n++] = 8 * d;
    if (budget_bytes < 0) dg.n = 0;
    const int blocks = admit_coop_blocks(n);
    void* args[] = {&a, &sc, &dg};
    const cudaError_t e = cudaLaunchCooperativeKernel(reinterpret_cast<void*>(admit_persistent_kernel), dim3(blocks),
                                                      dim3(256), args, 0, s);
    if (e != cudaSuccess) return fail(SKV_ERR_CUDA, "admit_codes: cooperative launch failed: %s", cudaGetErrorString(e));
    return check_launch("admit_persistent");
}

}  // extern "C"
