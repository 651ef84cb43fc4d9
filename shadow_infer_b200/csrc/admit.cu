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
#include <stddef.h>

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
__device__ __forceinline__ void sensitivity_d128_rows(const float* __restrict__ k, const float* __restrict__ v,
                                                      int B, int H, int S, int h, int t0, int lane,
                                                      float* __restrict__ sens) {
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

// Resident grid (a whole number of blocks per SM) walking the (head, 32-row chunk) items in
// head-major order, so that consecutive items read consecutive memory; 8 warps x RPW rows each.
template <int RPW>
__global__ void __launch_bounds__(256) sensitivity_d128_kernel(const float* __restrict__ k,
                                                               const float* __restrict__ v, int B, int H,
                                                               int S, float* __restrict__ sens) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nchunks = (S + 8 * RPW - 1) / (8 * RPW);
    const long long items = (long long)H * nchunks;
    for (long long it = blockIdx.x; it < items; it += gridDim.x) {
        const int h = (int)(it / nchunks);
        const int t0 = ((int)(it - (long long)h * nchunks) * 8 + warp) * RPW;
        if (t0 < S) sensitivity_d128_rows<RPW>(k, v, B, H, S, h, t0, lane, sens);
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

__device__ __forceinline__ bool eligible(const AdmitArgs& a, int64_t i) {
    if (i / a.H < a.sink) return false;
    if (a.prot && a.prot[i]) return false;
    return true;
}

// Unique, order-preserving key: score bits above the flat index (idx_bits >= log2(n)), so
// ascending keys are the reference's stable ascending-score order.
__device__ __forceinline__ unsigned long long entry_key(const AdmitArgs& a, int64_t i, int idx_bits) {
    const float imp = a.imp[i];
    const float s = (a.rd && a.sens) ? __fmul_rn(imp, a.sens[i]) : imp;
    return ((unsigned long long)score_bits(s) << idx_bits) | (unsigned long long)i;
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
// launch (one 1024-thread block per SM).  Keys are (score bits << idx_bits) | flat index, cut
// into 10-bit digits from the top.  Each pass histograms the candidates' weights per digit,
// together with their count and largest key, into its own global histogram (zeroed in-kernel
// before the first barrier); after a bounded grid barrier every block scans the same
// histogram and narrows the key prefix identically.  When the boundary bin holds a single
// candidate its key is that bin's largest key, so a phase usually ends after 2-3 passes.
// ---------------------------------------------------------------------------------------
constexpr int kAdmitThreads = 1024;
constexpr int kDigitBits = 10;
constexpr int kBins = 1 << kDigitBits;
constexpr int kAdmitMaxPasses = 7;                     // ceil(64 / 10)
static_assert(kBins == kAdmitThreads, "one histogram bin per thread");

struct AdmitScratch {
    long long sums[4];                                 // predicted0, predicted_final, evicted, -
    unsigned bar_count, bar_gen;
    int err, pad;
    unsigned long long hist_k[2 * kAdmitMaxPasses][kBins];
    unsigned int hist_c[2 * kAdmitMaxPasses][5][kBins];   // candidates per (weight class, digit)
};
constexpr size_t kAdmitHeaderBytes = offsetof(AdmitScratch, hist_k);

struct AdmitPlanDigits {
    int lo[kAdmitMaxPasses];                           // lowest key bit of each digit
    int width[kAdmitMaxPasses];                        // bits in each digit (<= kDigitBits)
    int n;
    int idx_bits;
};

__device__ __forceinline__ bool grid_barrier(AdmitScratch* sc, unsigned nblocks, unsigned& epoch) {
    return grid_sync_bounded(&sc->bar_count, &sc->err, nblocks, epoch);
}

__device__ __forceinline__ long long block_sum_ll(long long v, long long* s_red) {
    v = warp_sum_ll(v);
    if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = v;
    __syncthreads();
    long long t = 0;
    if (threadIdx.x == 0)
        for (int k = 0; k < kAdmitThreads / 32; ++k) t += s_red[k];
    __syncthreads();
    return t;
}

// KC > 0: each thread keeps its (at most KC) entries' keys and codes in registers for all
// passes; KC == 0: entries are re-read from memory in every pass (inputs beyond KC per thread).
template <int KC>
__global__ void __launch_bounds__(kAdmitThreads, 1)
    admit_persistent_kernel(AdmitArgs a, AdmitScratch* sc, AdmitPlanDigits dg) {
    __shared__ unsigned long long s_k[kBins];
    __shared__ unsigned int s_c[5][kBins];             // candidates per (weight class, digit)
    __shared__ unsigned long long s_before;
    __shared__ long long s_red[kAdmitThreads / 32];
    __shared__ AdmitHeader st;                         // identical in every block
    __shared__ int s_found;
    const unsigned nblocks = gridDim.x;
    const int tid = threadIdx.x;
    const int64_t stride = (int64_t)nblocks * kAdmitThreads;
    const unsigned long long idx_mask = dg.idx_bits >= 64 ? ~0ull : ((1ull << dg.idx_bits) - 1ull);
    bool ok = true;
    unsigned epoch = 0;                                // grid barriers passed

    // zero this launch's histograms (ordered before their first use by the barrier below)
    {
        unsigned long long* k = &sc->hist_k[0][0];
        unsigned int* c = &sc->hist_c[0][0][0];
        for (int64_t i = blockIdx.x * (int64_t)kAdmitThreads + tid; i < 2 * kAdmitMaxPasses * kBins; i += stride) {
            k[i] = 0;
#pragma unroll
            for (int q = 0; q < 5; ++q) c[q * 2 * kAdmitMaxPasses * kBins + i] = 0;
        }
    }
    // predicted bytes of the input codes (and the register cache of keys and codes)
    constexpr int KR = KC > 0 ? KC : 1;
    unsigned long long ck[KR];
    int cb[KR];                                        // base code (low byte) | 0x100 if a candidate
    const int64_t gtid = blockIdx.x * (int64_t)kAdmitThreads + tid;
    long long acc = 0;
    if (KC > 0) {
#pragma unroll
        for (int r = 0; r < KR; ++r) {
            const int64_t i = gtid + r * stride;
            ck[r] = 0;
            cb[r] = 0;
            if (i < a.n) {
                const int base = a.codes[i];
                acc += cost_of(a, base);
                cb[r] = (base & 0xFF);
                if (eligible(a, i)) {
                    ck[r] = entry_key(a, i, dg.idx_bits);
                    cb[r] |= 0x100;
                }
            }
        }
    } else {
        for (int64_t i = gtid; i < a.n; i += stride) acc += cost_of(a, a.codes[i]);
    }
    acc = block_sum_ll(acc, s_red);
    if (tid == 0 && acc) atomicAdd((unsigned long long*)&sc->sums[0], (unsigned long long)acc);
    ok = grid_barrier(sc, nblocks, epoch);
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
        hist_id = phase * kAdmitMaxPasses;
        for (int pass = 0; pass < dg.n && ok; ++pass, ++hist_id) {
            if (phase == 0 ? st.a_done : st.b_done) break;
            const int lo = dg.lo[pass];
            const unsigned long long dmask = (1ull << dg.width[pass]) - 1ull;
            s_k[tid] = 0;
#pragma unroll
            for (int q = 0; q < 5; ++q) s_c[q][tid] = 0;
            __syncthreads();
            const unsigned long long prefix = st.prefix, pmask = st.pmask;
            // a candidate's weight depends only on its weight class: the base code in the
            // downgrade phase (ladder saving wA), the code after it in the eviction phase
            // (entry cost), so the pass counts candidates per (class, digit).  Lanes with the
            // same (class, digit) are combined and one of them adds to the shared count.
            auto add = [&](bool cand, unsigned long long key, int base) {
                int cls = -1;
                if (cand && (key & pmask) == prefix) {
                    cls = phase == 0 ? base : code_after_a(st, base, key);
                    if (cls < 0 || cls > 4 || (phase == 0 ? a.wA[cls] : a.cost[cls]) == 0) cls = -1;
                }
                const unsigned active = __ballot_sync(0xffffffffu, cls >= 0);
                if (cls < 0) return;
                const int d = (int)((key >> lo) & dmask);
                const unsigned grp = __match_any_sync(active, d * 8 + cls);
                if ((threadIdx.x & 31) == __ffs(grp) - 1) {
                    atomicAdd(&s_c[cls][d], (unsigned)__popc(grp));
                    // a bin's key is read only when it ends up with ONE candidate in the whole
                    // grid, and then this is the only write to it
                    s_k[d] = key;
                }
            };
            if (KC > 0) {
#pragma unroll
                for (int r = 0; r < KR; ++r) add((cb[r] & 0x100) != 0, ck[r], (int)(int8_t)(cb[r] & 0xFF));
            } else {
                // warp-uniform trip count: rounds start at the warp's first entry
                const int64_t w0 = gtid - (tid & 31);
                for (int64_t i0 = w0; i0 < a.n; i0 += stride) {
                    const int64_t i = i0 + (tid & 31);
                    const bool cand = i < a.n && eligible(a, i);
                    add(cand, cand ? entry_key(a, i, dg.idx_bits) : 0ull, cand ? (int)a.codes[i] : 0);
                }
            }
            __syncthreads();
            {
                unsigned tot = 0;
#pragma unroll
                for (int q = 0; q < 5; ++q) {
                    const unsigned c = s_c[q][tid];
                    if (c) atomicAdd(&sc->hist_c[hist_id][q][tid], c);
                    tot += c;
                }
                if (tot == 1) sc->hist_k[hist_id][tid] = s_k[tid];   // see above
            }
            ok = grid_barrier(sc, nblocks, epoch);
            if (!ok) break;
            // every block scans the same global histogram: inclusive prefix of the weights
            long long v = 0;
            unsigned cnt_t = 0;
#pragma unroll
            for (int q = 0; q < 5; ++q) {
                const unsigned c = __ldcg(&sc->hist_c[hist_id][q][tid]);
                cnt_t += c;
                v += (long long)c * (phase == 0 ? a.wA[q] : a.cost[q]);
            }
            s_c[0][tid] = cnt_t;
            s_k[tid] = __ldcg(&sc->hist_k[hist_id][tid]);
            const int lane = tid & 31, wid = tid >> 5;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const long long y = __shfl_up_sync(0xffffffffu, v, o);
                if (lane >= o) v += y;
            }
            if (lane == 31) s_red[wid] = v;
            if (tid == 0) s_found = kBins;
            __syncthreads();
            if (wid == 0) {
                long long t = s_red[lane];
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const long long y = __shfl_up_sync(0xffffffffu, t, o);
                    if (lane >= o) t += y;
                }
                s_red[lane] = t;
            }
            __syncthreads();
            const long long cum = v + (wid > 0 ? s_red[wid - 1] : 0);
            const long long total = s_red[kAdmitThreads / 32 - 1];
            const long long rem = st.rem;
            if (cum >= rem) atomicMin(&s_found, tid);
            __syncthreads();
            const int d = s_found;
            // the bin just below the boundary bin holds the weight before it
            if (d < kBins && tid == (d > 0 ? d - 1 : 0)) s_before = d > 0 ? (unsigned long long)cum : 0ull;
            __syncthreads();
            if (tid == 0) {
                if (d == kBins) {
                    // all candidate weight falls short: the whole candidate list is consumed
                    if (phase == 0) {
                        st.a_notenough = 1;
                        st.a_done = 1;
                        st.predicted_a = st.predicted0 - total;
                    } else {
                        st.b_notenough = 1;
                        st.b_done = 1;
                    }
                } else {
                    const long long before = (long long)s_before;
                    st.rem = rem - before;
                    st.prefix |= (unsigned long long)d << lo;
                    st.pmask |= dmask << lo;
                    const unsigned cnt = s_c[0][d];
                    if (cnt == 1 || pass == dg.n - 1) {
                        const unsigned long long key = cnt == 1 ? s_k[d] : st.prefix;
                        if (phase == 0) {
                            const int64_t idx = (int64_t)(key & idx_mask);
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
    auto apply = [&](int64_t i, int base, bool cand, unsigned long long key) {
        int code = base;
        if (ok && cand && (st.a_active || st.b_active)) {
            code = code_after_a(st, base, key);
            if (st.b_active && (st.b_notenough || key <= st.b_key)) {
                if (code != 4) ++ev;
                code = 4;
            }
        }
        a.out[i] = (int8_t)code;
        pred += cost_of(a, code);
    };
    if (KC > 0) {
#pragma unroll
        for (int r = 0; r < KR; ++r) {
            const int64_t i = gtid + r * stride;
            if (i < a.n) apply(i, (int)(int8_t)(cb[r] & 0xFF), (cb[r] & 0x100) != 0, ck[r]);
        }
    } else {
        for (int64_t i = gtid; i < a.n; i += stride) {
            const bool cand = eligible(a, i);
            apply(i, a.codes[i], cand, cand ? entry_key(a, i, dg.idx_bits) : 0ull);
        }
    }
    pred = block_sum_ll(pred, s_red);
    ev = block_sum_ll(ev, s_red);
    if (tid == 0) {
        if (pred) atomicAdd((unsigned long long*)&sc->sums[1], (unsigned long long)pred);
        if (ev) atomicAdd((unsigned long long*)&sc->sums[2], (unsigned long long)ev);
    }
    const bool fin = grid_barrier(sc, nblocks, epoch);
    if (blockIdx.x == 0 && tid == 0) {
        const bool good = ok && fin && __ldcg(&sc->err) == 0;
        a.result[0] = good ? (long long)__ldcg((const unsigned long long*)&sc->sums[1]) : -1;
        a.result[1] = good ? (long long)__ldcg((const unsigned long long*)&sc->sums[2]) : -1;
    }
}

// One block per SM (cooperative launch: all resident), fewer for small inputs.
static int admit_coop_blocks(int64_t n) {
    const int64_t want = (n + kAdmitThreads - 1) / kAdmitThreads;
    const int64_t cap = sm_count();
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
        const long long items = (long long)H * ((S + 8 * kRPW - 1) / (8 * kRPW));
        static int per_sm = 0;          // resident blocks per SM (same on every B200 of the process)
        if (per_sm == 0 && (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, sensitivity_d128_kernel<kRPW>,
                                                                           256, 0) != cudaSuccess || per_sm < 1))
            per_sm = 4;
        const long long resident = (long long)sm_count() * per_sm;
        const int grid = (int)(items < resident ? items : resident);
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
    // the header (sums, barrier, error word); the kernel zeroes its own histograms
    if (cudaMemsetAsync(sc, 0, kAdmitHeaderBytes, s) != cudaSuccess)
        return fail(SKV_ERR_CUDA, "admit_codes: memset failed");
    // 10-bit digits of the (32 + idx_bits)-bit key, from the top
    int idx_bits = 0;
    while (idx_bits < 32 && ((int64_t)1 << idx_bits) < n) ++idx_bits;
    AdmitPlanDigits dg;
    dg.idx_bits = idx_bits;
    dg.n = 0;
    for (int hi = 32 + idx_bits; hi > 0 && dg.n < kAdmitMaxPasses; hi -= kDigitBits) {
        const int lo = hi > kDigitBits ? hi - kDigitBits : 0;
        dg.lo[dg.n] = lo;
        dg.width[dg.n] = hi - lo;
        ++dg.n;
    }
    if (budget_bytes < 0) dg.n = 0;
    const int blocks = admit_coop_blocks(n);
    void* args[] = {&a, &sc, &dg};
    constexpr int kCache = 8;
    void* fn = n <= (int64_t)blocks * kAdmitThreads * kCache ? reinterpret_cast<void*>(admit_persistent_kernel<kCache>)
                                                             : reinterpret_cast<void*>(admit_persistent_kernel<0>);
    const cudaError_t e = cudaLaunchCooperativeKernel(fn, dim3(blocks),
                                                      dim3(kAdmitThreads), args, 0, s);
    if (e != cudaSuccess) return fail(SKV_ERR_CUDA, "admit_codes: cooperative launch failed: %s", cudaGetErrorString(e));
    return check_launch("admit_persistent");
}

}  // extern "C"
