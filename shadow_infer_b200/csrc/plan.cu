// Precision coding and plan bucketing.
//
//  * skv_allocate_codes      -- threshold bands of ShadowKVAgent.allocate_precision_codes
//                               (shadowinfer/shadowkv/shadowkv_agent.py:1028-1059), float64
//                               comparisons as in the reference.
//  * skv_predict_codes_bytes -- sum of per-code costs (rd_allocator.py:170-187).
//  * skv_plan_bucket         -- PrecisionPlan.from_codes (precision_plan.py:113-177): a
//                               stable 5-way partition of the int8 [S,H] codes in
//                               token-major order plus the reuse-list compaction, done as
//                               a tile-count pass, a scan over the tile counts and a
//                               scatter pass (no sort).
#include <math.h>

#include <mutex>

#include "skv_common.cuh"

namespace skv {

// ---------------------------------------------------------------------------------------
// allocate_precision_codes
// ---------------------------------------------------------------------------------------
__global__ void allocate_codes_kernel(const float* __restrict__ imp, int64_t n, double t32,
                                      double t16, double t8, int8_t* __restrict__ codes) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        const double s = (double)imp[i];
        codes[i] = s >= t32 ? 0 : (s >= t16 ? 1 : (s >= t8 ? 2 : 3));
    }
}

// ---------------------------------------------------------------------------------------
// predict_codes_bytes
// ---------------------------------------------------------------------------------------
struct CostTable {
    long long c[5];
};

__host__ inline CostTable cost_table(int B, int D, int group_size) {
    // int(entry_bytes(...)) of rd_allocator.py:26-44, K+V incl. scales
    CostTable t;
    const int g = (group_size > 0 && D % group_size == 0) ? group_size : D;
    const double i4 = ((double)B * D / 2.0 + (double)B * (D / g) * 4) * 2.0;
    t.c[0] = (long long)((double)B * D * 4 * 2.0);
    t.c[1] = (long long)((double)B * D * 2 * 2.0);
    t.c[2] = (long long)(((double)B * D + (double)B * 4) * 2.0);
    t.c[3] = (long long)i4;
    t.c[4] = 0;
    return t;
}

__global__ void predict_bytes_kernel(const int8_t* __restrict__ codes, int64_t n, CostTable ct,
                                     long long* __restrict__ out) {
    long long acc = 0;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int c = codes[i];
        acc += (c >= 0 && c <= 4) ? ct.c[c] : 0;
    }
    acc = warp_sum_ll(acc);
    __shared__ long long s[32];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    if (lane == 0) s[w] = acc;
    __syncthreads();
    if (w == 0) {
        acc = lane < (int)(blockDim.x >> 5) ? s[lane] : 0;
        acc = warp_sum_ll(acc);
        if (lane == 0 && acc) atomicAdd((unsigned long long*)out, (unsigned long long)acc);
    }
}

// ---------------------------------------------------------------------------------------
// plan bucketing
// ---------------------------------------------------------------------------------------
constexpr int kPlanThreads = 256;
constexpr int kPlanItems = 8;
constexpr int kPlanTile = kPlanThreads * kPlanItems;   // entries per block
constexpr int kPlanCats = 6;                           // codes 0..4 + reuse
constexpr int kPlanStride = 8;                         // ints per tile in scratch

__device__ __forceinline__ void load_items(const int8_t* __restrict__ codes,
                                           const uint8_t* __restrict__ reuse, int64_t n,
                                           int64_t first, int (&c)[kPlanItems],
                                           int (&r)[kPlanItems]) {
#pragma unroll
    for (int j = 0; j < kPlanItems; ++j) {
        const int64_t i = first + j;
        c[j] = i < n ? (int)codes[i] : -1;
        r[j] = (reuse != nullptr && i < n) ? (reuse[i] != 0) : 0;
    }
}

// Packs three 16-bit counters per 64-bit word: categories {0,1,2} and {3,4,5}.
__device__ __forceinline__ void pack_counts(const int (&c)[kPlanItems], const int (&r)[kPlanItems],
                                            unsigned long long& lo, unsigned long long& hi) {
    lo = 0;
    hi = 0;
#pragma unroll
    for (int j = 0; j < kPlanItems; ++j) {
        const int cc = c[j];
        if (cc >= 0 && cc < 3) lo += 1ull << (16 * cc);
        else if (cc >= 3 && cc <= 4) hi += 1ull << (16 * (cc - 3));
        if (r[j]) hi += 1ull << 32;
    }
}

__device__ __forceinline__ int field(unsigned long long lo, unsigned long long hi, int cat) {
    return cat < 3 ? (int)((lo >> (16 * cat)) & 0xffff) : (int)((hi >> (16 * (cat - 3))) & 0xffff);
}

// Block-wide exclusive scan of two packed words; returns block totals too.
__device__ __forceinline__ void block_scan2(unsigned long long& lo, unsigned long long& hi,
                                            unsigned long long& tot_lo, unsigned long long& tot_hi) {
    __shared__ unsigned long long s_lo[kPlanThreads / 32], s_hi[kPlanThreads / 32];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    unsigned long long il = lo, ih = hi;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const unsigned long long a = __shfl_up_sync(0xffffffffu, il, o);
        const unsigned long long b = __shfl_up_sync(0xffffffffu, ih, o);
        if (lane >= o) {
            il += a;
            ih += b;
        }
    }
    if (lane == 31) {
        s_lo[w] = il;
        s_hi[w] = ih;
    }
    __syncthreads();
    unsigned long long wl = 0, wh = 0, tl = 0, th = 0;
#pragma unroll
    for (int k = 0; k < kPlanThreads / 32; ++k) {
        if (k < w) {
            wl += s_lo[k];
            wh += s_hi[k];
        }
        tl += s_lo[k];
        th += s_hi[k];
    }
    lo = wl + il - lo;
    hi = wh + ih - hi;
    tot_lo = tl;
    tot_hi = th;
    __syncthreads();
}

__global__ void __launch_bounds__(kPlanThreads) plan_count_kernel(
    const int8_t* __restrict__ codes, const uint8_t* __restrict__ reuse, int64_t n,
    int* __restrict__ tile_counts) {
    int c[kPlanItems], r[kPlanItems];
    const int64_t first = (int64_t)blockIdx.x * kPlanTile + (int64_t)threadIdx.x * kPlanItems;
    load_items(codes, reuse, n, first, c, r);
    unsigned long long lo, hi, tl, th;
    pack_counts(c, r, lo, hi);
    block_scan2(lo, hi, tl, th);
    if (threadIdx.x < kPlanCats) tile_counts[(int64_t)blockIdx.x * kPlanStride + threadIdx.x] =
        field(tl, th, threadIdx.x);
}

// Exclusive prefix over the tiles of each category's tile count, in place, and the category
// totals into counts[0..5]: one block walks the tiles kPrefixThreads at a time with a running
// carry, so every scatter block then reads its own prefix only (the work grows linearly with
// the number of tiles).  Prefixes stay below 2^31: S*H is limited to 2^29.
constexpr int kPrefixThreads = 1024;
__global__ void __launch_bounds__(kPrefixThreads) plan_prefix_kernel(int* __restrict__ tile_counts, int num_tiles,
                                                                      int64_t* __restrict__ counts) {
    __shared__ int s_warp[kPrefixThreads / 32][kPlanCats];
    __shared__ int s_chunk[kPlanCats];
    __shared__ long long s_carry[kPlanCats];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    if (threadIdx.x < kPlanCats) s_carry[threadIdx.x] = 0;
    __syncthreads();
    for (int base = 0; base < num_tiles; base += kPrefixThreads) {
        const int t = base + threadIdx.x;
        int v[kPlanCats], incl[kPlanCats];
#pragma unroll
        for (int k = 0; k < kPlanCats; ++k) {
            v[k] = t < num_tiles ? tile_counts[(int64_t)t * kPlanStride + k] : 0;
            incl[k] = v[k];
        }
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
#pragma unroll
            for (int k = 0; k < kPlanCats; ++k) {
                const int x = __shfl_up_sync(0xffffffffu, incl[k], o);
                if (lane >= o) incl[k] += x;
            }
        }
        if (lane == 31) {
#pragma unroll
            for (int k = 0; k < kPlanCats; ++k) s_warp[w][k] = incl[k];
        }
        __syncthreads();
        if (w == 0) {
            // exclusive scan of the 32 warp totals of each category; the last lane holds the chunk total
#pragma unroll
            for (int k = 0; k < kPlanCats; ++k) {
                const int x = s_warp[lane][k];
                int y = x;
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const int z = __shfl_up_sync(0xffffffffu, y, o);
                    if (lane >= o) y += z;
                }
                s_warp[lane][k] = y - x;
                if (lane == 31) s_chunk[k] = y;
            }
        }
        __syncthreads();
        if (t < num_tiles) {
#pragma unroll
            for (int k = 0; k < kPlanCats; ++k)
                tile_counts[(int64_t)t * kPlanStride + k] = (int)(s_carry[k] + s_warp[w][k] + incl[k] - v[k]);
        }
        __syncthreads();
        if (threadIdx.x < kPlanCats) s_carry[threadIdx.x] += s_chunk[threadIdx.x];
        __syncthreads();
    }
    if (threadIdx.x < kPlanCats) counts[threadIdx.x] = s_carry[threadIdx.x];
}

__global__ void __launch_bounds__(kPlanThreads) plan_scatter_kernel(
    const int8_t* __restrict__ codes, const uint8_t* __restrict__ reuse, int64_t n, int S, int H,
    const int* __restrict__ tile_prefix, const int64_t* __restrict__ counts, int64_t* __restrict__ flat_out,
    int32_t* __restrict__ slot_out, int64_t* __restrict__ reuse_out) {
    // 1. this tile's prefix per category (plan_prefix_kernel) and the bucket bases in flat_out
    __shared__ long long s_prefix[kPlanCats], s_base[kPlanCats];
    if (threadIdx.x < kPlanCats) s_prefix[threadIdx.x] = tile_prefix[(int64_t)blockIdx.x * kPlanStride + threadIdx.x];
    if (threadIdx.x == 0) {
        long long base = 0;
        for (int k = 0; k < 5; ++k) {
            s_base[k] = base;
            base += counts[k];
        }
        s_base[5] = 0;
    }
    __syncthreads();

    // 2. rank of every item within its category
    int c[kPlanItems], r[kPlanItems];
    const int64_t first = (int64_t)blockIdx.x * kPlanTile + (int64_t)threadIdx.x * kPlanItems;
    load_items(codes, reuse, n, first, c, r);
    unsigned long long lo, hi, tl, th;
    pack_counts(c, r, lo, hi);
    block_scan2(lo, hi, tl, th);
    int run[kPlanCats];
#pragma unroll
    for (int k = 0; k < kPlanCats; ++k) run[k] = field(lo, hi, k);
#pragma unroll
    for (int j = 0; j < kPlanItems; ++j) {
        const int64_t i = first + j;
        if (i >= n) break;
        const int64_t t = i / H, h = i - t * H;
        const int64_t f = h * S + t;
        const int cc = c[j];
        int32_t slot = -1;
        if (cc >= 0 && cc <= 4) {
            const long long pos = s_prefix[cc] + run[cc];
            run[cc] += 1;
            flat_out[s_base[cc] + pos] = f;
            if (cc < 4) slot = make_slot((int32_t)pos, cc);
        }
        if (slot_out) slot_out[i] = slot;
        if (r[j]) {
            reuse_out[s_prefix[5] + run[5]] = f;
            run[5] += 1;
        }
    }
}

// ---------------------------------------------------------------------------------------
// Allocation-free variant of the plan bucketing: the tile counts live in a fixed array in
// the library's device memory instead of a caller-provided scratch buffer.
// ---------------------------------------------------------------------------------------
constexpr int kStaticPlanTiles = 2048;                                  // tiles of kPlanTile entries
constexpr int64_t kStaticPlanMaxEntries = (int64_t)kStaticPlanTiles * kPlanTile;   // 4,194,304
static __device__ __align__(256) int g_plan_static_scratch[kStaticPlanTiles * kPlanStride];  // 64 KiB

// Device address of g_plan_static_scratch for the current device.  The host-side symbol is
// only a stand-in, so the address is looked up once per device (with that device current)
// and cached.
static int static_plan_scratch(int** out) {
    static std::mutex mu;
    static int* cached[64] = {nullptr};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
        return fail(SKV_ERR_CUDA, "plan_bucket_static: no current CUDA device");
    std::lock_guard<std::mutex> lock(mu);
    if (cached[dev] == nullptr) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_plan_static_scratch);
        if (e != cudaSuccess || p == nullptr)
            return fail(SKV_ERR_CUDA, "plan_bucket_static: cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
        cached[dev] = reinterpret_cast<int*>(p);
    }
    *out = cached[dev];
    return SKV_OK;
}

}  // namespace skv

using namespace skv;

extern "C" {

int64_t skv_plan_static_max_entries(void) { return kStaticPlanMaxEntries; }

int skv_plan_bucket_static(const int8_t* codes, const uint8_t* reuse_mask, int S, int H, int64_t* flat_out,
                           int32_t* slot_out, int64_t* reuse_flat_out, int64_t* counts, void* stream) {
    if (S <= 0 || H <= 0)
        return fail(SKV_ERR_INVALID_ARGUMENT, "seq_len and num_heads must be positive, got %d, %d", S, H);
    if (!codes || !flat_out || !counts || (reuse_mask && !reuse_flat_out))
        return fail(SKV_ERR_INVALID_ARGUMENT, "plan_bucket_static: null pointer");
    const int64_t n = (int64_t)S * H;
    if (n > kStaticPlanMaxEntries)
        return fail(SKV_ERR_TOO_LARGE,
                    "plan_bucket_static: seq_len*num_heads = %lld exceeds the %lld entries its fixed "
                    "device scratch covers; use skv_plan_bucket with a caller-provided scratch",
                    (long long)n, (long long)kStaticPlanMaxEntries);
    int* tc = nullptr;
    int st = static_plan_scratch(&tc);
    if (st) return st;
    // every tile count the prefix and scatter kernels read is written by plan_count_kernel of
    // the same call, so nothing left over from an earlier call needs clearing
    const int tiles = (int)((n + kPlanTile - 1) / kPlanTile);
    cudaStream_t s = as_stream(stream);
    plan_count_kernel<<<tiles, kPlanThreads, 0, s>>>(codes, reuse_mask, n, tc);
    st = check_launch("plan_count");
    if (st) return st;
    plan_prefix_kernel<<<1, kPrefixThreads, 0, s>>>(tc, tiles, counts);
    st = check_launch("plan_prefix");
    if (st) return st;
    plan_scatter_kernel<<<tiles, kPlanThreads, 0, s>>>(codes, reuse_mask, n, S, H, tc, counts, flat_out, slot_out,
                                                       reuse_flat_out);
    return check_launch("plan_scatter");
}


int skv_allocate_codes(const float* importance, int64_t n, int mode, int8_t* codes, void* stream) {
    if (n < 0) return fail(SKV_ERR_INVALID_ARGUMENT, "allocate_codes: negative size");
    if (n == 0) return SKV_OK;
    if (!importance || !codes) return fail(SKV_ERR_INVALID_ARGUMENT, "allocate_codes: null pointer");
    const double adj = mode == 0 ? -0.1 : (mode == 2 ? 0.1 : 0.0);
    const double t32 = fmax(0.0, 0.8 + adj), t16 = fmax(0.0, 0.5 + adj), t8 = fmax(0.0, 0.2 + adj);
    const int threads = 256;
    const int64_t want = (n + threads - 1) / threads;
    const int blocks = (int)(want < (int64_t)sm_count() * 16 ? want : (int64_t)sm_count() * 16);
    allocate_codes_kernel<<<blocks, threads, 0, as_stream(stream)>>>(importance, n, t32, t16, t8, codes);
    return check_launch("allocate_codes");
}

int skv_predict_codes_bytes(const int8_t* codes, int64_t n, int batch, int head_dim, int group_size,
                            int64_t* out, void* stream) {
    if (!out || (n > 0 && !codes)) return fail(SKV_ERR_INVALID_ARGUMENT, "predict_codes_bytes: null pointer");
    cudaStream_t s = as_stream(stream);
    if (cudaMemsetAsync(out, 0, sizeof(int64_t), s) != cudaSuccess)
        return fail(SKV_ERR_CUDA, "predict_codes_bytes: memset failed");
    if (n == 0) return SKV_OK;
    const int threads = 256;
    const int64_t want = (n + threads - 1) / threads;
    const int blocks = (int)(want < (int64_t)sm_count() * 8 ? want : (int64_t)sm_count() * 8);
    predict_bytes_kernel<<<blocks, threads, 0, s>>>(codes, n, cost_table(batch, head_dim, group_size),
                                                   (long long*)out);
    return check_launch("predict_codes_bytes");
}

size_t skv_plan_scratch_bytes(int S, int H) {
    const int64_t n = (int64_t)S * H;
    const int64_t tiles = (n + kPlanTile - 1) / kPlanTile;
    return (size_t)(tiles > 0 ? tiles : 1) * kPlanStride * sizeof(int);
}

int skv_plan_bucket(const int8_t* codes, const uint8_t* reuse_mask, int S, int H, int64_t* flat_out,
                    int32_t* slot_out, int64_t* reuse_flat_out, int64_t* counts, void* scratch,
                    size_t scratch_bytes, void* stream) {
    if (S <= 0 || H <= 0)
        return fail(SKV_ERR_INVALID_ARGUMENT, "seq_len and num_heads must be positive, got %d, %d", S, H);
    if (!codes || !flat_out || !counts || !scratch || (reuse_mask && !reuse_flat_out))
        return fail(SKV_ERR_INVALID_ARGUMENT, "plan_bucket: null pointer");
    const int64_t n = (int64_t)S * H;
    if (n > (int64_t(1) << 29)) return fail(SKV_ERR_TOO_LARGE, "plan_bucket: S*H above 2^29");
    if (scratch_bytes < skv_plan_scratch_bytes(S, H))
        return fail(SKV_ERR_SCRATCH, "plan_bucket: scratch %zu < %zu", scratch_bytes,
                    skv_plan_scratch_bytes(S, H));
    const int tiles = (int)((n + kPlanTile - 1) / kPlanTile);
    cudaStream_t s = as_stream(stream);
    int* tc = reinterpret_cast<int*>(scratch);
    plan_count_kernel<<<tiles, kPlanThreads, 0, s>>>(codes, reuse_mask, n, tc);
    int st = check_launch("plan_count");
    if (st) return st;
    plan_prefix_kernel<<<1, kPrefixThreads, 0, s>>>(tc, tiles, counts);
    st = check_launch("plan_prefix");
    if (st) return st;
    plan_scatter_kernel<<<tiles, kPlanThreads, 0, s>>>(codes, reuse_mask, n, S, H, tc, counts, flat_out, slot_out,
                                                       reuse_flat_out);
    return check_launch("plan_scatter");
}

}  // extern "C"
