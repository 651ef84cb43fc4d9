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
//    is found.  Each pass is one launch; the last block of a pass (ticket counter, no
//    spin-wait) scans the 256-bin histogram and narrows the key prefix.  A final pass
//    writes the new codes, the predicted bytes and the eviction count.
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

struct AdmitState : AdmitHeader {
    unsigned long long hist[256];
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

// Decision after the downgrade phase: predicted bytes and whether eviction runs.
__device__ void start_phase_b(const AdmitArgs& a, AdmitState* st, long long predicted_a) {
    st->predicted_a = predicted_a;
    st->b_active = (a.allow_evict && predicted_a > a.budget) ? 1 : 0;
    st->rem = predicted_a - a.budget;
    st->prefix = 0;
    st->pmask = 0;
}

// Block-wide search of the first histogram bin whose inclusive prefix reaches `rem`.
// Runs in the last block of a pass; all threads participate.
template <int PHASE>
__device__ void finish_pass(const AdmitArgs& a, AdmitState* st, int shift, int last_pass) {
    __shared__ long long s_inc[256];
    __shared__ int s_found;
    const int tid = threadIdx.x;
    long long hv = 0;
    if (tid < 256) hv = (long long)__ldcg(&st->hist[tid]);
    if (tid < 256) s_inc[tid] = hv;
    if (tid == 0) s_found = 256;
    __syncthreads();
    for (int o = 1; o < 256; o <<= 1) {
        long long add = (tid < 256 && tid >= o) ? s_inc[tid - o] : 0;
        __syncthreads();
        if (tid < 256) s_inc[tid] += add;
        __syncthreads();
    }
    const long long rem = st->rem;
    if (tid < 256 && s_inc[tid] >= rem) atomicMin(&s_found, tid);
    __syncthreads();
    if (tid == 0) {
        const int d = s_found;
        if (d == 256) {
            // total weight below the requirement: the whole candidate list is consumed
            const long long total = s_inc[255];
            if (PHASE == 0) {
                st->a_notenough = 1;
                st->a_done = 1;
                start_phase_b(a, st, st->predicted0 - total);
            } else {
                st->b_notenough = 1;
                st->b_done = 1;
            }
        } else {
            const long long before = d > 0 ? s_inc[d - 1] : 0;
            st->rem = rem - before;
            st->prefix |= (unsigned long long)d << shift;
            st->pmask |= 0xFFull << shift;
            if (last_pass) {
                const unsigned long long key = st->prefix;
                if (PHASE == 0) {
                    const int64_t idx = (int64_t)(key & 0xFFFFFFFFull);
                    const int base = a.codes[idx];
                    const long long r = st->rem;  // remaining excess at the boundary entry
                    const long long s1 = base < 3 ? a.delta[base] : 0;
                    const int n1 = base < 3 ? base + 1 : base;
                    const long long s2 = n1 < 3 ? a.delta[n1] : 0;
                    const int n2 = n1 < 3 ? n1 + 1 : n1;
                    int nc = base;
                    if (base != 4) nc = r <= s1 ? n1 : (r <= s1 + s2 ? n2 : 3);
                    st->a_key = key;
                    st->a_newcode = nc;
                    st->a_done = 1;
                    const long long consumed = (st->predicted0 - a.budget) - r;
                    start_phase_b(a, st, st->predicted0 - consumed - (a.cost[base] - a.cost[nc]));
                } else {
                    st->b_key = key;
                    st->b_done = 1;
                }
            }
        }
    }
    __syncthreads();
    if (tid < 256) st->hist[tid] = 0;
    if (tid == 0) st->counter = 0;
}

template <int PHASE>
__global__ void __launch_bounds__(256) admit_pass_kernel(AdmitArgs a, AdmitState* st, int shift, int last_pass) {
    __shared__ unsigned long long s_hist[256];
    __shared__ bool s_last;
    const AdmitHeader snap = *static_cast<const AdmitHeader*>(st);
    if (PHASE == 0 && (!snap.a_active || snap.a_done)) return;
    if (PHASE == 1 && (!snap.b_active || snap.b_done)) return;
    s_hist[threadIdx.x] = 0;
    __syncthreads();
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < a.n; i += (int64_t)gridDim.x * blockDim.x) {
        if (!eligible(a, i)) continue;
        const unsigned long long key = entry_key(a, i);
        if ((key & snap.pmask) != snap.prefix) continue;
        const int base = a.codes[i];
        long long w;
        if (PHASE == 0) w = (base >= 0 && base <= 4) ? a.wA[base] : 0;
        else w = cost_of(a, code_after_a(snap, base, key));
        if (w == 0) continue;
        atomicAdd(&s_hist[(key >> shift) & 0xFF], (unsigned long long)w);
    }
    __syncthreads();
    const unsigned long long hv = s_hist[threadIdx.x];
    if (hv) atomicAdd(&st->hist[threadIdx.x], hv);
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) s_last = atomicAdd(&st->counter, 1u) == gridDim.x - 1;
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    finish_pass<PHASE>(a, st, shift, last_pass);
}

__global__ void __launch_bounds__(256) admit_init_kernel(AdmitArgs a, AdmitState* st) {
    __shared__ long long s_red[8];
    __shared__ bool s_last;
    long long acc = 0;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < a.n; i += (int64_t)gridDim.x * blockDim.x)
        acc += cost_of(a, a.codes[i]);
    acc = warp_sum_ll(acc);
    if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = acc;
    __syncthreads();
    if (threadIdx.x == 0) {
        long long t = 0;
        for (int k = 0; k < 8; ++k) t += s_red[k];
        if (t) atomicAdd((unsigned long long*)&st->predicted0, (unsigned long long)t);
        __threadfence();
        s_last = atomicAdd(&st->counter, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (!s_last || threadIdx.x != 0) return;
    __threadfence();
    const long long p0 = (long long)atomicAdd((unsigned long long*)&st->predicted0, 0ull);
    st->a_active = (a.budget >= 0 && p0 > a.budget) ? 1 : 0;
    st->rem = p0 - a.budget;
    st->prefix = 0;
    st->pmask = 0;
    st->predicted_a = p0;
    st->b_active = 0;
    st->counter = 0;
}

__global__ void __launch_bounds__(256) admit_apply_kernel(AdmitArgs a, AdmitState* st) {
    __shared__ long long s_p[8], s_e[8];
    __shared__ bool s_last;
    const AdmitHeader snap = *static_cast<const AdmitHeader*>(st);
    long long pred = 0, ev = 0;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < a.n; i += (int64_t)gridDim.x * blockDim.x) {
        const int base = a.codes[i];
        int code = base;
        if (eligible(a, i) && (snap.a_active || snap.b_active)) {
            const unsigned long long key = entry_key(a, i);
            code = code_after_a(snap, base, key);
            if (snap.b_active && (snap.b_notenough || key <= snap.b_key)) {
                if (code != 4) ++ev;
                code = 4;
            }
        }
        a.out[i] = (int8_t)code;
        pred += cost_of(a, code);
    }
    pred = warp_sum_ll(pred);
    ev = warp_sum_ll(ev);
    if ((threadIdx.x & 31) == 0) {
        s_p[threadIdx.x >> 5] = pred;
        s_e[threadIdx.x >> 5] = ev;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        long long tp = 0, te = 0;
        for (int k = 0; k < 8; ++k) {
            tp += s_p[k];
            te += s_e[k];
        }
        if (tp) atomicAdd((unsigned long long*)&st->predicted_final, (unsigned long long)tp);
        if (te) atomicAdd((unsigned long long*)&st->evicted, (unsigned long long)te);
        __threadfence();
        s_last = atomicAdd(&st->counter, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (!s_last || threadIdx.x != 0) return;
    __threadfence();
    a.result[0] = (long long)atomicAdd((unsigned long long*)&st->predicted_final, 0ull);
    a.result[1] = (long long)atomicAdd((unsigned long long*)&st->evicted, 0ull);
    st->counter = 0;
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
    return sizeof(AdmitState);
}

int skv_admit_codes(const int8_t* codes_in, int8_t* codes_out, const float* importance, const float* sensitivity,
                    const uint8_t* protected_mask, int S, int H, int64_t budget_bytes, int batch, int head_dim,
                    int group_size, int sink_tokens, int rd_allocation, int allow_eviction, void* scratch,
                    size_t scratch_bytes, int64_t* result, void* stream) {
    if (S <= 0 || H <= 0) return fail(SKV_ERR_INVALID_ARGUMENT, "admit_codes: bad shape");
    if (!codes_in || !codes_out || !importance || !scratch || !result)
        return fail(SKV_ERR_INVALID_ARGUMENT, "admit_codes: null pointer");
    if (scratch_bytes < sizeof(AdmitState))
        return fail(SKV_ERR_SCRATCH, "admit_codes: scratch %zu < %zu", scratch_bytes, sizeof(AdmitState));
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
    AdmitState* st = reinterpret_cast<AdmitState*>(scratch);
    if (cudaMemsetAsync(st, 0, sizeof(AdmitState), s) != cudaSuccess)
        return fail(SKV_ERR_CUDA, "admit_codes: memset failed");
    const int64_t want = (n + 1023) / 1024;
    const int blocks = (int)(want < (int64_t)sm_count() * 2 ? (want > 0 ? want : 1) : (int64_t)sm_count() * 2);
    admit_init_kernel<<<blocks, 256, 0, s>>>(a, st);
    int stc = check_launch("admit_init");
    if (stc) return stc;
    // digit shifts: 4 score digits, then enough index digits to cover n-1
    int idx_bits = 0;
    while (idx_bits < 63 && ((int64_t)1 << idx_bits) < n) ++idx_bits;
    const int idx_digits = (idx_bits + 7) / 8;
    int shifts[8];
    int np = 0;
    for (int d = 3; d >= 0; --d) shifts[np++] = 32 + 8 * d;
    for (int d = idx_digits - 1; d >= 0; --d) shifts[np++] = 8 * d;
    if (budget_bytes >= 0) {
        for (int phase = 0; phase < (allow_eviction ? 2 : 1); ++phase) {
            for (int i = 0; i < np; ++i) {
                if (phase == 0) admit_pass_kernel<0><<<blocks, 256, 0, s>>>(a, st, shifts[i], i == np - 1);
                else admit_pass_kernel<1><<<blocks, 256, 0, s>>>(a, st, shifts[i], i == np - 1);
                stc = check_launch("admit_pass");
                if (stc) return stc;
            }
        }
    }
    admit_apply_kernel<<<blocks, 256, 0, s>>>(a, st);
    return check_launch("admit_apply");
}

}  // extern "C"
