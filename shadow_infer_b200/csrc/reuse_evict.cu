// Reuse scatter and in-bucket eviction.
//
//  * skv_apply_reuse   -- PackedKVCache.apply_reuse_mask (shadowinfer/shadowkv/
//                         packed_kv_cache.py:753-854): per current entry with the reuse
//                         flag, copy the previous step's row (payload + scales) when the
//                         previous cache holds the entry in the same precision; count the
//                         cross-precision ones.  One warp per 32 entries; the selected rows'
//                         16-byte chunks are spread over the lanes through a warp prefix sum.
//  * skv_evict_count / skv_evict_compact -- PackedKVCache.evict (packed_kv_cache.py:666-740):
//                         stable compaction of every bucket without the evicted (t,h): a
//                         tile-count pass, then a scan + row-move pass into new buckets.
#include "skv_common.cuh"

namespace skv {

__device__ __forceinline__ bool aligned16(const void* a, const void* b, const void* c, const void* d) {
    return ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b) | reinterpret_cast<uintptr_t>(c) |
             reinterpret_cast<uintptr_t>(d)) & 15) == 0;
}

// One warp per 32 consecutive entries; the reuse flag and both slots of an entry are loaded
// together.  The payload rows to copy, of every precision, are cut into 16-byte chunks numbered
// through a warp prefix sum of the rows' chunk counts; each pass hands every lane kChunks chunks
// of K and of V, all loaded before the first store, so one warp keeps up to 2 * 32 * kChunks
// loads in flight whatever the precision mix, and 64 registers allow 32 warps per SM.  A lane
// copies its own entry's scales (at most 8 floats per row, as float4) after the payload.  Rows that are not whole 16-byte
// chunks at 16-byte aligned addresses take a per-row warp copy instead.
constexpr int kChunks = 2;   // 16-byte chunks of K and of V per lane and pass

__global__ void __launch_bounds__(256, 4) reuse_kernel(const __grid_constant__ Buckets cur,
                                                       const int32_t* __restrict__ cur_slot, int S,
                                                       const __grid_constant__ Buckets prev,
                                                       const int32_t* __restrict__ prev_slot,
                                                    int S_prev, const uint8_t* __restrict__ mask, int B,
                                                    int H, int D, int NG, long long* __restrict__ stats) {
    const int lane = threadIdx.x & 31;
    const int64_t n = (int64_t)S * H;
    const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    long long applied = 0, skipped = 0;
    for (int64_t base = (((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5) * 32; base < n;
         base += nwarps * 32) {
        const int64_t e = base + lane;
        int32_t cs = -1, ps = -1;
        bool flag = false;
        if (e < n) {
            const int64_t t = e / H;
            flag = mask[e] != 0;
            cs = cur_slot[e];
            ps = t < S_prev ? prev_slot[e] : -1;           // same H: entry (t, h) sits at t*H + h
        }
        bool copy = false;
        if (flag && cs >= 0 && ps >= 0) {
            if (slot_code(ps) == slot_code(cs)) copy = true;
            else skipped += 1;
        }
        applied += copy ? 1 : 0;
        if (!__any_sync(0xffffffffu, copy)) continue;
        const int code = copy ? slot_code(cs) : 0;
        const int64_t rb = copy ? payload_row_bytes(code, B, D) : 0;
        const int64_t sf = copy ? scale_row_floats(code, B, D, NG) : 0;
        const int64_t cp = slot_pos(cs), pp = slot_pos(ps);
        const skv_bucket& cb = cur.b[code];
        const skv_bucket& pb = prev.b[code];
        // payload: whole 16-byte chunks at aligned addresses go through the chunk passes
        const bool chunked = copy && (rb & 15) == 0 && aligned16(cb.k, cb.v, pb.k, pb.v);
        const int nch = chunked ? (int)(rb >> 4) : 0;
        int incl = nch;                                      // inclusive prefix over the lanes
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int x = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += x;
        }
        const int total = __shfl_sync(0xffffffffu, incl, 31);
        for (int j0 = 0; j0 < total; j0 += 32 * kChunks) {
            uint4 a[kChunks], b[kChunks];
            uint8_t* dk[kChunks];
            uint8_t* dv[kChunks];
#pragma unroll
            for (int u = 0; u < kChunks; ++u) {
                const int j = j0 + u * 32 + lane;
                // the row holding chunk j: the first lane whose inclusive prefix exceeds j
                int r = 0;
#pragma unroll
                for (int step = 16; step > 0; step >>= 1)
                    if (__shfl_sync(0xffffffffu, incl, r + step - 1) <= j) r += step;
                const int r_incl = __shfl_sync(0xffffffffu, incl, r);
                const int r_n = __shfl_sync(0xffffffffu, nch, r);
                const int r_code = __shfl_sync(0xffffffffu, code, r);
                const int32_t r_cp = __shfl_sync(0xffffffffu, (int32_t)cp, r);
                const int32_t r_pp = __shfl_sync(0xffffffffu, (int32_t)pp, r);
                dk[u] = nullptr;
                dv[u] = nullptr;
                if (j < total) {
                    const int64_t rbr = (int64_t)r_n * 16;
                    const int64_t off = (int64_t)(j - (r_incl - r_n)) * 16;
                    const skv_bucket& cbr = cur.b[r_code];
                    const skv_bucket& pbr = prev.b[r_code];
                    a[u] = __ldg(reinterpret_cast<const uint4*>(reinterpret_cast<const uint8_t*>(pbr.k) + r_pp * rbr + off));
                    b[u] = __ldg(reinterpret_cast<const uint4*>(reinterpret_cast<const uint8_t*>(pbr.v) + r_pp * rbr + off));
                    dk[u] = reinterpret_cast<uint8_t*>(cbr.k) + r_cp * rbr + off;
                    dv[u] = reinterpret_cast<uint8_t*>(cbr.v) + r_cp * rbr + off;
                }
            }
#pragma unroll
            for (int u = 0; u < kChunks; ++u)
                if (dk[u] != nullptr) {
                    *reinterpret_cast<uint4*>(dk[u]) = a[u];
                    *reinterpret_cast<uint4*>(dv[u]) = b[u];
                }
        }
        // scales: this lane's own row (after the payload passes, so that their registers are free)
        const bool svec = copy && sf > 0 && (sf & 3) == 0 && sf <= 8 &&
                          aligned16(pb.scale_k + pp * sf, pb.scale_v + pp * sf, cb.scale_k + cp * sf,
                                    cb.scale_v + cp * sf);
        float4 k0 = make_float4(0.f, 0.f, 0.f, 0.f), v0 = k0, k1 = k0, v1 = k0;
        if (svec) {
            const float4* ssk = reinterpret_cast<const float4*>(pb.scale_k + pp * sf);
            const float4* ssv = reinterpret_cast<const float4*>(pb.scale_v + pp * sf);
            k0 = __ldg(ssk);
            v0 = __ldg(ssv);
            if (sf > 4) {
                k1 = __ldg(ssk + 1);
                v1 = __ldg(ssv + 1);
            }
        }
        if (svec) {
            float4* dsk = reinterpret_cast<float4*>(cb.scale_k + cp * sf);
            float4* dsv = reinterpret_cast<float4*>(cb.scale_v + cp * sf);
            dsk[0] = k0;
            dsv[0] = v0;
            if (sf > 4) {
                dsk[1] = k1;
                dsv[1] = v1;
            }
        } else if (copy) {
            for (int64_t i = 0; i < sf; ++i) {
                cb.scale_k[cp * sf + i] = pb.scale_k[pp * sf + i];
                cb.scale_v[cp * sf + i] = pb.scale_v[pp * sf + i];
            }
        }
        // rows the chunk passes do not cover: one warp copy per row
        unsigned todo = __ballot_sync(0xffffffffu, copy && !chunked);
        while (todo) {
            const int src = __ffs(todo) - 1;
            todo &= todo - 1;
            const int c2 = __shfl_sync(0xffffffffu, code, src);
            const int64_t cpos = __shfl_sync(0xffffffffu, (int32_t)cp, src);
            const int64_t ppos = __shfl_sync(0xffffffffu, (int32_t)pp, src);
            const int64_t rb2 = payload_row_bytes(c2, B, D);
            warp_copy(reinterpret_cast<uint8_t*>(cur.b[c2].k) + cpos * rb2,
                      reinterpret_cast<const uint8_t*>(prev.b[c2].k) + ppos * rb2, rb2, lane);
            warp_copy(reinterpret_cast<uint8_t*>(cur.b[c2].v) + cpos * rb2,
                      reinterpret_cast<const uint8_t*>(prev.b[c2].v) + ppos * rb2, rb2, lane);
        }
    }
    if (!stats) return;                                 // statistics not requested
    applied = warp_sum_ll(applied);
    skipped = warp_sum_ll(skipped);
    if (lane == 0) {
        if (applied) atomicAdd((unsigned long long*)&stats[0], (unsigned long long)applied);
        if (skipped) atomicAdd((unsigned long long*)&stats[1], (unsigned long long)skipped);
    }
}

// ---------------------------------------------------------------------------------------
// evict
// ---------------------------------------------------------------------------------------
constexpr int kEvThreads = 256;
constexpr int kEvItems = 4;
constexpr int kEvTile = kEvThreads * kEvItems;

__device__ __forceinline__ bool evicted_flag(const uint8_t* __restrict__ mask, int64_t f, int S, int H) {
    const int64_t h = f / S, t = f - h * S;
    return mask[t * H + h] != 0;
}

// Block-wide exclusive scan of one int per thread; returns the block total.
__device__ __forceinline__ int block_exclusive_scan(int x, int& total) {
    __shared__ int s_w[kEvThreads / 32];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    int inc = x;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += y;
    }
    if (lane == 31) s_w[w] = inc;
    __syncthreads();
    int before = 0;
    total = 0;
#pragma unroll
    for (int k = 0; k < kEvThreads / 32; ++k) {
        if (k < w) before += s_w[k];
        total += s_w[k];
    }
    __syncthreads();
    return before + inc - x;
}

__global__ void __launch_bounds__(kEvThreads) evict_count_kernel(Buckets src, const uint8_t* __restrict__ mask,
                                                                 int S, int H, int max_tiles,
                                                                 int* __restrict__ tile_kept,
                                                                 long long* __restrict__ kept) {
    const int p = blockIdx.y;
    const int64_t count = src.b[p].count;
    const int64_t first = (int64_t)blockIdx.x * kEvTile;
    if (first >= count) return;
    int keep = 0;
    for (int j = 0; j < kEvItems; ++j) {
        const int64_t i = first + (int64_t)threadIdx.x * kEvItems + j;
        if (i < count && !evicted_flag(mask, src.b[p].flat[i], S, H)) ++keep;
    }
    int total;
    block_exclusive_scan(keep, total);
    if (threadIdx.x == 0) {
        tile_kept[(int64_t)p * max_tiles + blockIdx.x] = total;
        const int64_t in_tile = count - first < kEvTile ? count - first : kEvTile;
        atomicAdd((unsigned long long*)&kept[p], (unsigned long long)total);
        atomicAdd((unsigned long long*)&kept[4], (unsigned long long)(in_tile - total));
    }
}

// Rows of `cpr` 16-byte chunks (K and V tensors alike) of tile entries li -> new[li] (-1: not
// kept): chunk c of the tile is chunk c % cpr of entry c / cpr; each thread takes every
// kEvThreads-th chunk, four at a time with their loads issued first.
__device__ __forceinline__ void copy_rows16(uint8_t* __restrict__ dk, uint8_t* __restrict__ dv,
                                            const uint8_t* __restrict__ sk, const uint8_t* __restrict__ sv,
                                            int cpr, int64_t first, int in_tile, const int32_t* s_new) {
    const int total = in_tile * cpr;
    for (int c0 = threadIdx.x; c0 < total; c0 += 4 * kEvThreads) {
        uint4 a[4], b[4];
        int64_t d_off[4];
        bool ok[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int c = c0 + u * kEvThreads;
            const int li = c < total ? c / cpr : 0;
            const int32_t np = c < total ? s_new[li] : -1;
            ok[u] = np >= 0;
            d_off[u] = 0;
            if (ok[u]) {
                const int off = (c - li * cpr) * 16;
                const int64_t s_off = (first + li) * (int64_t)cpr * 16 + off;
                d_off[u] = (int64_t)np * cpr * 16 + off;
                a[u] = __ldg(reinterpret_cast<const uint4*>(sk + s_off));
                b[u] = __ldg(reinterpret_cast<const uint4*>(sv + s_off));
            }
        }
#pragma unroll
        for (int u = 0; u < 4; ++u)
            if (ok[u]) {
                *reinterpret_cast<uint4*>(dk + d_off[u]) = a[u];
                *reinterpret_cast<uint4*>(dv + d_off[u]) = b[u];
            }
    }
}

__global__ void __launch_bounds__(kEvThreads) evict_compact_kernel(
    Buckets src, Buckets dst, const uint8_t* __restrict__ mask, int32_t* __restrict__ slot, int B, int S,
    int H, int D, int NG, int max_tiles, const int* __restrict__ tile_kept) {
    const int p = blockIdx.y;
    const int64_t count = src.b[p].count;
    const int64_t first = (int64_t)blockIdx.x * kEvTile;
    // a bucket that loses nothing is passed with dst.count == src.count and left untouched
    if (first >= count || dst.b[p].count == count) return;
    __shared__ int s_red[kEvThreads / 32];
    __shared__ int32_t s_new[kEvTile];
    // prefix of kept entries in earlier tiles of this bucket
    int pre = 0;
    for (int t = threadIdx.x; t < (int)blockIdx.x; t += kEvThreads) pre += tile_kept[(int64_t)p * max_tiles + t];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) pre += __shfl_xor_sync(0xffffffffu, pre, o);
    if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = pre;
    __syncthreads();
    int prefix = 0;
    for (int k = 0; k < kEvThreads / 32; ++k) prefix += s_red[k];
    __syncthreads();

    int64_t f[kEvItems];
    bool keep[kEvItems];
    int nkeep = 0;
    for (int j = 0; j < kEvItems; ++j) {
        const int64_t i = first + (int64_t)threadIdx.x * kEvItems + j;
        keep[j] = false;
        f[j] = -1;
        if (i < count) {
            f[j] = src.b[p].flat[i];
            keep[j] = !evicted_flag(mask, f[j], S, H);
            nkeep += keep[j];
        }
    }
    int total;
    int run = block_exclusive_scan(nkeep, total) + prefix;
    for (int j = 0; j < kEvItems; ++j) {
        const int li = threadIdx.x * kEvItems + j;
        s_new[li] = -1;
        if (f[j] < 0) continue;
        const int64_t h = f[j] / S, t = f[j] - h * S;
        if (keep[j]) {
            dst.b[p].flat[run] = f[j];
            slot[t * H + h] = make_slot(run, p);
            s_new[li] = run;
            ++run;
        } else {
            slot[t * H + h] = -1;
        }
    }
    __syncthreads();
    // move the kept rows: the 16-byte chunks of every row of the tile are spread over the
    // block's threads, four chunk copies in flight per thread (loads before stores)
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int64_t rb = payload_row_bytes(p, B, D);
    const int64_t sf = scale_row_floats(p, B, D, NG);
    const int in_tile = (int)(count - first < kEvTile ? count - first : kEvTile);
    const skv_bucket& sb = src.b[p];
    const skv_bucket& db = dst.b[p];
    if ((rb & 15) == 0 && aligned16(sb.k, sb.v, db.k, db.v)) {
        copy_rows16(reinterpret_cast<uint8_t*>(db.k), reinterpret_cast<uint8_t*>(db.v),
                    reinterpret_cast<const uint8_t*>(sb.k), reinterpret_cast<const uint8_t*>(sb.v), (int)(rb / 16),
                    first, in_tile, s_new);
    } else {
        for (int li = w; li < in_tile; li += kEvThreads / 32) {
            const int32_t np = s_new[li];
            if (np < 0) continue;
            const int64_t op = first + li;
            warp_copy(reinterpret_cast<uint8_t*>(db.k) + np * rb, reinterpret_cast<const uint8_t*>(sb.k) + op * rb,
                      rb, lane);
            warp_copy(reinterpret_cast<uint8_t*>(db.v) + np * rb, reinterpret_cast<const uint8_t*>(sb.v) + op * rb,
                      rb, lane);
        }
    }
    if (sf) {
        if (((sf * 4) & 15) == 0 && aligned16(sb.scale_k, sb.scale_v, db.scale_k, db.scale_v)) {
            copy_rows16(reinterpret_cast<uint8_t*>(db.scale_k), reinterpret_cast<uint8_t*>(db.scale_v),
                        reinterpret_cast<const uint8_t*>(sb.scale_k), reinterpret_cast<const uint8_t*>(sb.scale_v),
                        (int)(sf * 4 / 16), first, in_tile, s_new);
        } else {
            const int total = in_tile * (int)sf;
            for (int e = threadIdx.x; e < total; e += kEvThreads) {
                const int li = e / (int)sf;
                const int32_t np = s_new[li];
                if (np < 0) continue;
                const int64_t i = e - (int64_t)li * sf;
                const int64_t op = first + li;
                db.scale_k[np * sf + i] = sb.scale_k[op * sf + i];
                db.scale_v[np * sf + i] = sb.scale_v[op * sf + i];
            }
        }
    }
}

static int64_t max_count(const skv_bucket* b) {
    int64_t m = 0;
    for (int p = 0; p < kNumBuckets; ++p) m = b[p].count > m ? b[p].count : m;
    return m;
}

}  // namespace skv

using namespace skv;

extern "C" {

int skv_apply_reuse(const skv_bucket* cur, const int32_t* cur_slot, int S, const skv_bucket* prev,
                    const int32_t* prev_slot, int S_prev, const uint8_t* reuse_mask, int B, int H, int D,
                    int int4_group, int64_t* stats, void* stream) {
    if (!cur || !prev || !cur_slot || !prev_slot || !reuse_mask)
        return fail(SKV_ERR_INVALID_ARGUMENT, "apply_reuse: null pointer");
    if (B <= 0 || H <= 0 || S <= 0 || S_prev <= 0 || D <= 0)
        return fail(SKV_ERR_INVALID_ARGUMENT, "apply_reuse: bad shape");
    cudaStream_t s = as_stream(stream);
    if (stats && cudaMemsetAsync(stats, 0, 2 * sizeof(int64_t), s) != cudaSuccess)
        return fail(SKV_ERR_CUDA, "apply_reuse: memset failed");
    const int G = int4_group > 0 && D % int4_group == 0 ? int4_group : D;
    Buckets c, p;
    for (int i = 0; i < kNumBuckets; ++i) {
        c.b[i] = cur[i];
        p.b[i] = prev[i];
    }
    const int64_t n = (int64_t)S * H;
    const int64_t want = (n + 255) / 256;
    const int blocks = (int)(want < (int64_t)sm_count() * 8 ? want : (int64_t)sm_count() * 8);
    reuse_kernel<<<blocks > 0 ? blocks : 1, 256, 0, s>>>(c, cur_slot, S, p, prev_slot, S_prev, reuse_mask, B, H, D,
                                                         D / G, (long long*)stats);
    return check_launch("apply_reuse");
}

size_t skv_evict_scratch_bytes(int64_t max_bucket_entries) {
    const int64_t tiles = (max_bucket_entries + kEvTile - 1) / kEvTile;
    return (size_t)(tiles > 0 ? tiles : 1) * kNumBuckets * sizeof(int);
}

int skv_evict_count(const skv_bucket* src, const uint8_t* evict_mask, int S, int H, int64_t* kept,
                    void* scratch, size_t scratch_bytes, void* stream) {
    if (!src || !evict_mask || !kept || !scratch) return fail(SKV_ERR_INVALID_ARGUMENT, "evict_count: null pointer");
    if (S <= 0 || H <= 0) return fail(SKV_ERR_INVALID_ARGUMENT, "evict_count: bad shape");
    const int64_t m = max_count(src);
    if (scratch_bytes < skv_evict_scratch_bytes(m))
        return fail(SKV_ERR_SCRATCH, "evict_count: scratch %zu < %zu", scratch_bytes, skv_evict_scratch_bytes(m));
    cudaStream_t s = as_stream(stream);
    if (cudaMemsetAsync(kept, 0, 5 * sizeof(int64_t), s) != cudaSuccess)
        return fail(SKV_ERR_CUDA, "evict_count: memset failed");
    if (m == 0) return SKV_OK;
    Buckets b;
    for (int i = 0; i < kNumBuckets; ++i) b.b[i] = src[i];
    const int tiles = (int)((m + kEvTile - 1) / kEvTile);
    evict_count_kernel<<<dim3(tiles, kNumBuckets), kEvThreads, 0, s>>>(b, evict_mask, S, H, tiles,
                                                                       reinterpret_cast<int*>(scratch),
                                                                       (long long*)kept);
    return check_launch("evict_count");
}

int skv_evict_compact(const skv_bucket* src, const skv_bucket* dst, const uint8_t* evict_mask, int32_t* slot,
                      int B, int S, int H, int D, int int4_group, void* scratch, size_t scratch_bytes,
                      void* stream) {
    if (!src || !dst || !evict_mask || !slot || !scratch)
        return fail(SKV_ERR_INVALID_ARGUMENT, "evict_compact: null pointer");
    if (B <= 0 || S <= 0 || H <= 0 || D <= 0) return fail(SKV_ERR_INVALID_ARGUMENT, "evict_compact: bad shape");
    const int64_t m = max_count(src);
    if (scratch_bytes < skv_evict_scratch_bytes(m))
        return fail(SKV_ERR_SCRATCH, "evict_compact: scratch too small");
    if (m == 0) return SKV_OK;
    const int G = int4_group > 0 && D % int4_group == 0 ? int4_group : D;
    Buckets a, b;
    for (int i = 0; i < kNumBuckets; ++i) {
        a.b[i] = src[i];
        b.b[i] = dst[i];
    }
    const int tiles = (int)((m + kEvTile - 1) / kEvTile);
    evict_compact_kernel<<<dim3(tiles, kNumBuckets), kEvThreads, 0, as_stream(stream)>>>(
        a, b, evict_mask, slot, B, S, H, D, D / G, tiles, reinterpret_cast<const int*>(scratch));
    return check_launch("evict_compact");
}

}  // extern "C"
