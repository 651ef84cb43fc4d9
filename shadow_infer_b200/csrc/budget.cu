// Cross-layer budget enforcement: the device side of KVCacheManager.enforce_global_budget
// (shadowinfer/shadowkv/kv_cache_manager.py:129-200).
//
// The reference lists every non-sink (layer, token, head) of the layers that have an importance
// matrix, sorts the list stably by importance and evicts it from the front in batches,
// re-reading the manager's usage after each batch.  Only three quantities of that sorted list
// are ever needed -- how many bytes the first k entries free, for the few k the batch loop
// visits, and which entries the final k are -- so no sort is done here:
//
//  * skv_budget_candidates  writes one layer's candidates (token-major, then head, from the
//                           sink on) as a score and the resident bytes evicting it frees
//                           (0 for an entry not in the cache or a layer whose bytes the
//                           manager does not count);
//  * skv_rank_select        finds the k-th smallest (score, position) key and the summed
//                           bytes of the k smallest, in one cooperative launch of 10-bit
//                           radix passes (counts and bytes per digit);
//  * skv_mark_smallest      marks the candidates whose key is at most that k-th key.
//
// The key (score bits << idx_bits | position) is unique and orders exactly as the
// reference's stable sort of (score, list position).
#include <stddef.h>

#include "skv_common.cuh"

namespace skv {

struct Cost4 {
    long long c[4];
};

__global__ void budget_candidates_kernel(const float* __restrict__ imp, int S_m, int H_m,
                                         const int32_t* __restrict__ slot, int S_c, int H_c, int sink, Cost4 cost,
                                         float* __restrict__ score, long long* __restrict__ weight) {
    const int64_t n = (int64_t)(S_m - sink) * H_m;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int t = sink + (int)(i / H_m), h = (int)(i % H_m);
        score[i] = imp[(int64_t)t * H_m + h];
        long long w = 0;
        if (slot && t < S_c && h < H_c) {
            const int32_t s = slot[(int64_t)t * H_c + h];
            if (s >= 0) w = cost.c[slot_code(s)];
        }
        weight[i] = w;
    }
}

constexpr int kRsThreads = 1024;
constexpr int kRsDigitBits = 10;
constexpr int kRsBins = 1 << kRsDigitBits;
constexpr int kRsMaxPasses = 7;                        // ceil(64 / 10)
static_assert(kRsBins == kRsThreads, "one histogram bin per thread");

struct RankScratch {
    unsigned bar_count;
    int err;
    unsigned pad[2];
    unsigned long long hist_w[kRsMaxPasses][kRsBins];
    unsigned long long hist_k[kRsMaxPasses][kRsBins];
    unsigned int hist_c[kRsMaxPasses][kRsBins];
};
constexpr size_t kRankHeaderBytes = offsetof(RankScratch, hist_w);

struct RankDigits {
    int lo[kRsMaxPasses];
    int width[kRsMaxPasses];
    int n;
    int idx_bits;
};

__device__ __forceinline__ unsigned long long rank_key(const float* score, int64_t i, int idx_bits) {
    return ((unsigned long long)score_bits(score[i]) << idx_bits) | (unsigned long long)i;
}

// result[0] = summed weight of the k smallest keys, result[1] = the k-th smallest key;
// both -1 if a grid barrier failed.
__global__ void __launch_bounds__(kRsThreads, 1)
    rank_select_kernel(const float* __restrict__ score, const long long* __restrict__ weight, int64_t n, int64_t k,
                       RankScratch* sc, RankDigits dg, long long* result) {
    __shared__ unsigned long long s_w[kRsBins];
    __shared__ unsigned long long s_k[kRsBins];
    __shared__ unsigned int s_c[kRsBins];
    __shared__ long long s_red[kRsThreads / 32];
    __shared__ long long s_redw[kRsThreads / 32];
    __shared__ unsigned long long st_prefix, st_pmask, st_key;
    __shared__ long long st_krem, st_wacc, st_total;
    __shared__ int st_done, s_found;
    __shared__ long long s_before_c, s_before_w;
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    const unsigned nblocks = gridDim.x;
    const int64_t stride = (int64_t)nblocks * kRsThreads;
    const int64_t gtid = blockIdx.x * (int64_t)kRsThreads + tid;
    unsigned epoch = 0;
    for (int64_t i = gtid; i < (int64_t)kRsMaxPasses * kRsBins; i += stride) {
        (&sc->hist_w[0][0])[i] = 0;
        (&sc->hist_k[0][0])[i] = 0;
        (&sc->hist_c[0][0])[i] = 0;
    }
    if (tid == 0) {
        st_prefix = 0;
        st_pmask = 0;
        st_krem = k;
        st_wacc = 0;
        st_done = 0;
        st_key = 0;
        st_total = 0;
    }
    bool ok = grid_sync_bounded(&sc->bar_count, &sc->err, nblocks, epoch);
    for (int pass = 0; pass < dg.n && ok && !st_done; ++pass) {
        const int lo = dg.lo[pass];
        const unsigned long long dmask = (1ull << dg.width[pass]) - 1ull;
        s_w[tid] = 0;
        s_k[tid] = 0;
        s_c[tid] = 0;
        __syncthreads();
        const unsigned long long prefix = st_prefix, pmask = st_pmask;
        for (int64_t i = gtid; i < n; i += stride) {
            const unsigned long long key = rank_key(score, i, dg.idx_bits);
            if ((key & pmask) != prefix) continue;
            const int d = (int)((key >> lo) & dmask);
            atomicAdd(&s_c[d], 1u);
            atomicAdd(&s_w[d], (unsigned long long)weight[i]);
            s_k[d] = key;                              // read only for a bin with one key
        }
        __syncthreads();
        if (s_c[tid]) {
            atomicAdd(&sc->hist_c[pass][tid], s_c[tid]);
            atomicAdd(&sc->hist_w[pass][tid], s_w[tid]);
            if (s_c[tid] == 1) sc->hist_k[pass][tid] = s_k[tid];
        }
        ok = grid_sync_bounded(&sc->bar_count, &sc->err, nblocks, epoch);
        if (!ok) break;
        // every block scans the same histogram: inclusive prefix of counts and of weights
        const long long c = (long long)__ldcg(&sc->hist_c[pass][tid]);
        const long long w = (long long)__ldcg(&sc->hist_w[pass][tid]);
        s_c[tid] = (unsigned)c;
        s_w[tid] = (unsigned long long)w;
        s_k[tid] = __ldcg(&sc->hist_k[pass][tid]);
        long long vc = c, vw = w;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const long long yc = __shfl_up_sync(0xffffffffu, vc, o);
            const long long yw = __shfl_up_sync(0xffffffffu, vw, o);
            if (lane >= o) {
                vc += yc;
                vw += yw;
            }
        }
        if (lane == 31) {
            s_red[wid] = vc;
            s_redw[wid] = vw;
        }
        if (tid == 0) s_found = kRsBins;
        __syncthreads();
        if (wid == 0) {
            long long tc = s_red[lane], tw = s_redw[lane];
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const long long yc = __shfl_up_sync(0xffffffffu, tc, o);
                const long long yw = __shfl_up_sync(0xffffffffu, tw, o);
                if (lane >= o) {
                    tc += yc;
                    tw += yw;
                }
            }
            s_red[lane] = tc;
            s_redw[lane] = tw;
        }
        __syncthreads();
        const long long cum_c = vc + (wid > 0 ? s_red[wid - 1] : 0);
        const long long cum_w = vw + (wid > 0 ? s_redw[wid - 1] : 0);
        if (cum_c >= st_krem) atomicMin(&s_found, tid);
        __syncthreads();
        const int d = s_found;
        if (d < kRsBins && tid == d) {
            s_before_c = cum_c - c;
            s_before_w = cum_w - w;
        }
        __syncthreads();
        if (tid == 0) {
            if (d == kRsBins) {
                // k exceeds the candidates: cannot happen (the host checks k <= n)
                atomicExch(&sc->err, 2);
                st_done = 1;
            } else {
                st_krem -= s_before_c;
                st_wacc += s_before_w;
                st_prefix |= (unsigned long long)d << lo;
                st_pmask |= dmask << lo;
                if (s_c[d] == 1 || pass == dg.n - 1) {
                    st_key = s_c[d] == 1 ? s_k[d] : st_prefix;
                    st_total = st_wacc + (long long)s_w[d];
                    st_done = 1;
                }
            }
        }
        __syncthreads();
    }
    if (blockIdx.x == 0 && tid == 0) {
        const bool good = ok && st_done && __ldcg(&sc->err) == 0;
        result[0] = good ? st_total : -1;
        result[1] = good ? (long long)st_key : -1;
    }
}

__global__ void mark_smallest_kernel(const float* __restrict__ score, int64_t n, int idx_bits,
                                     const long long* __restrict__ result, uint8_t* __restrict__ mask) {
    const unsigned long long kth = (unsigned long long)result[1];
    const bool valid = result[0] >= 0;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        mask[i] = (valid && rank_key(score, i, idx_bits) <= kth) ? 1 : 0;
}

static int key_index_bits(int64_t n) {
    int b = 0;
    while (b < 32 && ((int64_t)1 << b) < n) ++b;
    return b;
}

}  // namespace skv

using namespace skv;

extern "C" {

int skv_budget_candidates(const float* importance, int S_m, int H_m, const int32_t* slot, int S_c, int H_c,
                          int sink_tokens, const int64_t* entry_cost, float* score, int64_t* weight, void* stream) {
    if (!importance || !score || !weight || !entry_cost)
        return fail(SKV_ERR_INVALID_ARGUMENT, "budget_candidates: null pointer");
    if (S_m <= 0 || H_m <= 0 || sink_tokens < 0) return fail(SKV_ERR_INVALID_ARGUMENT, "budget_candidates: bad shape");
    if (sink_tokens >= S_m) return SKV_OK;
    Cost4 cost;
    for (int c = 0; c < 4; ++c) cost.c[c] = entry_cost[c];
    const int64_t n = (int64_t)(S_m - sink_tokens) * H_m;
    const int64_t want = (n + 255) / 256;
    const int blocks = (int)(want < (int64_t)sm_count() * 8 ? want : (int64_t)sm_count() * 8);
    budget_candidates_kernel<<<blocks, 256, 0, as_stream(stream)>>>(importance, S_m, H_m, slot, S_c, H_c, sink_tokens,
                                                                   cost, score, reinterpret_cast<long long*>(weight));
    return check_launch("budget_candidates");
}

size_t skv_rank_select_scratch_bytes(int64_t n) {
    (void)n;
    return sizeof(RankScratch);
}

int skv_rank_select(const float* score, const int64_t* weight, int64_t n, int64_t k, void* scratch,
                    size_t scratch_bytes, int64_t* result, void* stream) {
    if (!score || !weight || !scratch || !result) return fail(SKV_ERR_INVALID_ARGUMENT, "rank_select: null pointer");
    if (n <= 0 || k < 1 || k > n) return fail(SKV_ERR_INVALID_ARGUMENT, "rank_select: need 1 <= k <= n");
    if (n >= ((int64_t)1 << 31)) return fail(SKV_ERR_TOO_LARGE, "rank_select: n above 2^31");
    if (scratch_bytes < sizeof(RankScratch))
        return fail(SKV_ERR_SCRATCH, "rank_select: scratch %zu < %zu", scratch_bytes, sizeof(RankScratch));
    cudaStream_t s = as_stream(stream);
    RankScratch* sc = reinterpret_cast<RankScratch*>(scratch);
    if (cudaMemsetAsync(sc, 0, kRankHeaderBytes, s) != cudaSuccess) return fail(SKV_ERR_CUDA, "rank_select: memset failed");
    RankDigits dg;
    dg.idx_bits = key_index_bits(n);
    dg.n = 0;
    for (int hi = 32 + dg.idx_bits; hi > 0 && dg.n < kRsMaxPasses; hi -= kRsDigitBits) {
        const int lo = hi > kRsDigitBits ? hi - kRsDigitBits : 0;
        dg.lo[dg.n] = lo;
        dg.width[dg.n] = hi - lo;
        ++dg.n;
    }
    const int64_t want = (n + kRsThreads - 1) / kRsThreads;
    const int blocks = (int)(want < (int64_t)sm_count() ? want : (int64_t)sm_count());
    long long* res = reinterpret_cast<long long*>(result);
    const long long* w = reinterpret_cast<const long long*>(weight);
    void* args[] = {(void*)&score, (void*)&w, &n, &k, &sc, &dg, &res};
    const cudaError_t e = cudaLaunchCooperativeKernel(reinterpret_cast<void*>(rank_select_kernel), dim3(blocks),
                                                      dim3(kRsThreads), args, 0, s);
    if (e != cudaSuccess) return fail(SKV_ERR_CUDA, "rank_select: cooperative launch failed: %s", cudaGetErrorString(e));
    return check_launch("rank_select");
}

int skv_mark_smallest(const float* score, int64_t n, const int64_t* result, uint8_t* mask, void* stream) {
    if (!score || !result || !mask) return fail(SKV_ERR_INVALID_ARGUMENT, "mark_smallest: null pointer");
    if (n <= 0) return fail(SKV_ERR_INVALID_ARGUMENT, "mark_smallest: bad size");
    if (n >= ((int64_t)1 << 31)) return fail(SKV_ERR_TOO_LARGE, "mark_smallest: n above 2^31");
    const int64_t want = (n + 255) / 256;
    const int blocks = (int)(want < (int64_t)sm_count() * 8 ? want : (int64_t)sm_count() * 8);
    mark_smallest_kernel<<<blocks, 256, 0, as_stream(stream)>>>(score, n, key_index_bits(n),
                                                               reinterpret_cast<const long long*>(result), mask);
    return check_launch("mark_smallest");
}

}  // extern "C"
