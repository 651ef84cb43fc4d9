// Page-table data plane of the paged KV store (shadowinfer/shadowkv/paged_kv_store.py).
//
// A page holds the rows of one precision for a run of consecutive tokens.  Its payload is a
// slab [B, H, cap, row] (row = D floats / D halves / D int8 / ceil(D/2) int4 bytes) plus, for
// int8 and int4, fp32 scales [B, H, cap] / [B, H, cap, D/G]; a page descriptor points at the
// slab's row that holds the page's first token (block (b, h) = 0), and `row_stride` (= cap)
// steps from one (b, h) block to the next.  The host keeps the descriptors of the pages in
// token order in a device page table.
//
//  * skv_paged_write        quantises source rows [B, H, T, D] straight into page slabs
//                           (append and rewrite_tokens), one warp per (page run, b, h, token)
//                           row, bit-identical to the reference's row-local Quantizer calls;
//                           it also stores the descriptors of the pages it wrote into the
//                           device page table, so appends need no separate table upload.
//  * skv_paged_gather       rebuilds dense fp32 K/V [B, H, S, D] in one launch over the page
//                           table: block (j, b*h, part) covers the hole before page j and
//                           page j itself, writing zeros into the hole and decoded rows
//                           elsewhere (8 values per thread when D and the int4 group allow).
//  * skv_paged_clear_heads  zeroes the rows of partially evicted (token, head) pairs
//                           (0x88 bytes for int4, which decode to 0).
#include <stddef.h>

#include <mutex>

#include "skv_common.cuh"

namespace skv {

static_assert(sizeof(skv_page_desc) == 64, "skv_page_desc is 64 bytes");
static_assert(sizeof(skv_page_write) == 88, "skv_page_write is 88 bytes");

constexpr int kPagedWarps = 8;
// Page writes travel as kernel parameters: up to 8 (704 B) for the usual append / rewrite,
// up to 256 (22.5 KB; parameters above 4 KB need CUDA 12.1+) for an append that opens many pages.
constexpr int kPagedFewWrites = 8;
constexpr int kPagedManyWrites = 256;

template <int N>
struct PagedWrites {
    skv_page_write w[N];
};

__host__ __device__ inline int64_t paged_row_bytes(int precision, int D) {
    switch (precision) {
        case 0: return (int64_t)D * 4;
        case 1: return (int64_t)D * 2;
        case 2: return D;
        default: return ((int64_t)D + 1) / 2;
    }
}

// One source row (D fp32 values) into one page row, by one warp.  `gsm`: this warp's
// ngroups words of shared memory (int4 groups that do not divide 32 lanes).
__device__ __forceinline__ void write_row(const float* __restrict__ src, void* dst, float* scale, int precision,
                                          int D, int G, int ngroups, unsigned* gsm, int lane) {
    if (precision == 0) {
        warp_copy(dst, src, (int64_t)D * 4, lane);
        return;
    }
    if (precision == 1) {
        __half* d = reinterpret_cast<__half*>(dst);
        for (int e = lane; e < D; e += kWarp) d[e] = __float2half_rn(__ldg(src + e));
        return;
    }
    if (precision == 2) {
        float m = 0.0f;
        for (int e = lane; e < D; e += kWarp) m = fmaxf(m, fabsf(__ldg(src + e)));
        m = warp_max(m);
        const float s = quant_scale(m, 127.0f), r = __frcp_rn(s);
        int8_t* d = reinterpret_cast<int8_t*>(dst);
        for (int e = lane; e < D; e += kWarp) d[e] = (int8_t)quant_value_fast(__ldg(src + e), s, r, -128, 127);
        if (lane == 0) scale[0] = s;
        return;
    }
    // int4: per-group absmax / 7; element pairs (2j, 2j+1) sit on lanes (even, odd) of one
    // 32-element chunk, so the odd lane's code reaches its partner with one shuffle.
    uint8_t* d = reinterpret_cast<uint8_t*>(dst);
    const bool lane_groups = (kWarp % G) == 0;   // groups are aligned lane blocks of G
    if (!lane_groups) {
        for (int g = lane; g < ngroups; g += kWarp) gsm[g] = 0u;
        __syncwarp();
        for (int e = lane; e < D; e += kWarp) atomicMax(gsm + e / G, __float_as_uint(fabsf(__ldg(src + e))));
        __syncwarp();
    }
    const int chunks = (D + kWarp - 1) / kWarp;
    for (int c = 0; c < chunks; ++c) {
        const int e = c * kWarp + lane;
        const float x = e < D ? __ldg(src + e) : 0.0f;
        const float m = lane_groups ? group_max(fabsf(x), G) : (e < D ? __uint_as_float(gsm[e / G]) : 0.0f);
        const float s = quant_scale(m, 7.0f);
        const int q = quant_value_fast(x, s, __frcp_rn(s), -8, 7);
        const int partner = __shfl_xor_sync(0xffffffffu, q, 1);
        if (e < D && (e & 1) == 0) {
            const unsigned lo = (e + 1 < D) ? (unsigned)(partner + 8) & 15u : 0u;
            d[e >> 1] = (uint8_t)((((unsigned)(q + 8) & 15u) << 4) | lo);
        }
        if (e < D && e % G == 0) scale[e / G] = s;
    }
    if (!lane_groups) __syncwarp();   // gsm is reused by the warp's next row
}

// grid (ceil(max_rows * B*H / 8), n_writes), 256 threads.
template <int N>
__global__ void __launch_bounds__(256) paged_write_kernel(const float* __restrict__ k, const float* __restrict__ v,
                                                         int BH, int64_t T_src, int D, int G,
                                                         const __grid_constant__ PagedWrites<N> ws,
                                                         skv_page_desc* __restrict__ table) {
    extern __shared__ unsigned paged_gsm[];
    const skv_page_write& w = ws.w[blockIdx.y];
    if (blockIdx.x == 0 && threadIdx.x == 0 && table != nullptr && w.table_pos >= 0) table[w.table_pos] = w.page;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t item = (int64_t)blockIdx.x * kPagedWarps + warp;
    if (item >= (int64_t)w.rows * BH) return;
    const int bh = (int)(item / w.rows), r = (int)(item % w.rows);
    const int p = w.page.precision;
    const int ngroups = D / G;
    const int64_t row = (int64_t)bh * w.page.row_stride + w.dst_row + r;
    const int64_t rb = paged_row_bytes(p, D);
    const int64_t srow = ((int64_t)bh * T_src + w.src_token + r) * D;
    const int64_t sstride = p == 3 ? ngroups : 1;
    unsigned* gsm = paged_gsm + warp * ngroups;
    write_row(k + srow, static_cast<uint8_t*>(w.page.k) + row * rb, w.page.scale_k ? w.page.scale_k + row * sstride : nullptr,
              p, D, G, ngroups, gsm, lane);
    write_row(v + srow, static_cast<uint8_t*>(w.page.v) + row * rb, w.page.scale_v ? w.page.scale_v + row * sstride : nullptr,
              p, D, G, ngroups, gsm, lane);
}

// Vector path (D in {32, 64, 128, 256}; int4 groups a multiple of V): the rows of one
// (write, b, h) run are contiguous in the source and in the page, so a warp walks them as one
// flat array, V consecutive values per lane and 32*V values (whole rows) per pass.  The lanes
// of a row (D/V of them) and of an int4 group (G/V) are aligned lane blocks, reduced with xor
// shuffles.  A warp takes PPW passes of K and V, all loads issued before the first store.
template <int V, int PPW, int N>
__global__ void __launch_bounds__(256) paged_write_vec_kernel(const float* __restrict__ k,
                                                             const float* __restrict__ v, int BH, int64_t T_src,
                                                             int D, int G, const __grid_constant__ PagedWrites<N> ws,
                                                             skv_page_desc* __restrict__ table) {
    const skv_page_write& w = ws.w[blockIdx.y];
    if (blockIdx.x == 0 && threadIdx.x == 0 && table != nullptr && w.table_pos >= 0) table[w.table_pos] = w.page;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t n_el = (int64_t)w.rows * D;
    const int passes = (int)((n_el + 32 * V - 1) / (32 * V));
    const int tasks_per_bh = (passes + PPW - 1) / PPW;
    const int64_t task = (int64_t)blockIdx.x * kPagedWarps + warp;
    if (task >= (int64_t)tasks_per_bh * BH) return;
    const int bh = (int)(task / tasks_per_bh), pass0 = (int)(task % tasks_per_bh) * PPW;
    const int p = w.page.precision;
    const int lpr = D / V;                     // lanes per row
    const int lpg = G / V;                     // lanes per int4 group
    const int ng = D / G;
    const int64_t src0 = ((int64_t)bh * T_src + w.src_token) * D;
    const int64_t row0 = (int64_t)bh * w.page.row_stride + w.dst_row;   // page row of the run's first token
    float xk[PPW][V], xv[PPW][V];
#pragma unroll
    for (int i = 0; i < PPW; ++i) {
        const int64_t e = (int64_t)(pass0 + i) * 32 * V + lane * V;
#pragma unroll
        for (int j = 0; j < V; j += 4) {
            float4 a = make_float4(0.f, 0.f, 0.f, 0.f), b = a;
            if (e < n_el) {
                a = __ldg(reinterpret_cast<const float4*>(k + src0 + e + j));
                b = __ldg(reinterpret_cast<const float4*>(v + src0 + e + j));
            }
            xk[i][j] = a.x; xk[i][j + 1] = a.y; xk[i][j + 2] = a.z; xk[i][j + 3] = a.w;
            xv[i][j] = b.x; xv[i][j + 1] = b.y; xv[i][j + 2] = b.z; xv[i][j + 3] = b.w;
        }
    }
#pragma unroll
    for (int t = 0; t < 2; ++t) {
        uint8_t* dst = static_cast<uint8_t*>(t ? w.page.v : w.page.k);
        float* sc = t ? w.page.scale_v : w.page.scale_k;
#pragma unroll
        for (int i = 0; i < PPW; ++i) {
            const float* x = t ? xv[i] : xk[i];
            const int64_t e = (int64_t)(pass0 + i) * 32 * V + lane * V;
            const bool on = e < n_el;
            const int64_t r = e / D;                   // run row
            const int col = (int)(e - r * D);
            const int64_t prow = row0 + r;            // page row (b, h block included)
            if (p == 0) {
                if (on) {
#pragma unroll
                    for (int j = 0; j < V; j += 4)
                        reinterpret_cast<float4*>(dst + (prow * D + col + j) * 4)[0] =
                            make_float4(x[j], x[j + 1], x[j + 2], x[j + 3]);
                }
            } else if (p == 1) {
                uint32_t h[V / 2];
#pragma unroll
                for (int j = 0; j < V / 2; ++j) {
                    const __half2 hv = __floats2half2_rn(x[2 * j], x[2 * j + 1]);
                    h[j] = *reinterpret_cast<const uint32_t*>(&hv);
                }
                if (on) {
                    if (V == 4) {
                        *reinterpret_cast<uint2*>(dst + (prow * D + col) * 2) = make_uint2(h[0], h[1]);
                    } else {
#pragma unroll
                        for (int j = 0; j < V / 2; j += 4)
                            *reinterpret_cast<uint4*>(dst + (prow * D + col + 2 * j) * 2) =
                                make_uint4(h[j], h[j + 1], h[j + 2], h[j + 3]);
                    }
                }
            } else {
                const bool i4 = p == 3;
                float m = 0.0f;
#pragma unroll
                for (int j = 0; j < V; ++j) m = fmaxf(m, fabsf(x[j]));
                m = group_max(m, i4 ? lpg : lpr);    // every lane runs the shuffles
                const float s = quant_scale(m, i4 ? 7.0f : 127.0f), rc = __frcp_rn(s);
                int q[V];
#pragma unroll
                for (int j = 0; j < V; ++j) q[j] = quant_value_fast(x[j], s, rc, i4 ? -8 : -128, i4 ? 7 : 127);
                if (on) {
                    if (!i4) {
#pragma unroll
                        for (int j = 0; j < V; j += 4) {
                            const uint32_t wd = ((uint32_t)(q[j] & 0xFF)) | ((uint32_t)(q[j + 1] & 0xFF) << 8) |
                                                ((uint32_t)(q[j + 2] & 0xFF) << 16) |
                                                ((uint32_t)(q[j + 3] & 0xFF) << 24);
                            *reinterpret_cast<uint32_t*>(dst + prow * D + col + j) = wd;
                        }
                        if (col == 0) sc[prow] = s;
                    } else {
                        uint32_t bytes[V / 2];
#pragma unroll
                        for (int j = 0; j < V / 2; ++j)
                            bytes[j] = (((uint32_t)(q[2 * j] + 8) & 15u) << 4) | ((uint32_t)(q[2 * j + 1] + 8) & 15u);
                        uint8_t* d = dst + (prow * D + col) / 2;
                        if (V == 4) {
                            *reinterpret_cast<uint16_t*>(d) = (uint16_t)(bytes[0] | (bytes[1] << 8));
                        } else {
#pragma unroll
                            for (int j = 0; j < V / 2; j += 4)
                                *reinterpret_cast<uint32_t*>(d + j) =
                                    bytes[j] | (bytes[j + 1] << 8) | (bytes[j + 2] << 16) | (bytes[j + 3] << 24);
                        }
                        if (col % G == 0) sc[prow * ng + col / G] = s;
                    }
                }
            }
        }
    }
}

// ------------------------------------------------------------------------------------ gather
__device__ __forceinline__ void st8(float* dst, const float (&x)[8]) {
    float4* d = reinterpret_cast<float4*>(dst);
    d[0] = make_float4(x[0], x[1], x[2], x[3]);
    d[1] = make_float4(x[4], x[5], x[6], x[7]);
}

// 8 consecutive values of one page row (D % 8 == 0; int4 groups of a multiple of 8).
__device__ __forceinline__ void decode8(const skv_page_desc& pg, bool is_v, int64_t row, int col, int D, int ngroups,
                                        int G, float (&x)[8]) {
    const uint8_t* base = static_cast<const uint8_t*>(is_v ? pg.v : pg.k);
    const float* sc = is_v ? pg.scale_v : pg.scale_k;
    const int p = pg.precision;
    if (p == 0) {
        const float4* s = reinterpret_cast<const float4*>(base + (row * D + col) * 4);
        const float4 a = __ldg(s), b = __ldg(s + 1);
        x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w; x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
    } else if (p == 1) {
        const uint4 u = __ldg(reinterpret_cast<const uint4*>(base + (row * D + col) * 2));
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
            x[2 * i] = f.x;
            x[2 * i + 1] = f.y;
        }
    } else if (p == 2) {
        const uint2 u = __ldg(reinterpret_cast<const uint2*>(base + row * D + col));
        const float s = __ldg(sc + row);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint32_t w = i < 4 ? u.x : u.y;
            x[i] = __fmul_rn((float)(int8_t)(w >> (8 * (i & 3))), s);
        }
    } else {
        const uint32_t w = __ldg(reinterpret_cast<const uint32_t*>(base + (row * D + col) / 2));
        const float s = __ldg(sc + row * ngroups + col / G);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t byte = (w >> (8 * i)) & 0xFFu;
            x[2 * i] = __fmul_rn((float)((int)(byte >> 4) - 8), s);
            x[2 * i + 1] = __fmul_rn((float)((int)(byte & 15u) - 8), s);
        }
    }
}

// One value of a page row, any D and group.
__device__ __forceinline__ float decode1(const skv_page_desc& pg, bool is_v, int64_t row, int col, int D, int ngroups,
                                         int G) {
    const uint8_t* base = static_cast<const uint8_t*>(is_v ? pg.v : pg.k);
    const float* sc = is_v ? pg.scale_v : pg.scale_k;
    switch (pg.precision) {
        case 0: return __ldg(reinterpret_cast<const float*>(base) + row * D + col);
        case 1: return __half2float(reinterpret_cast<const __half*>(base)[row * D + col]);
        case 2: return __fmul_rn((float)reinterpret_cast<const int8_t*>(base)[row * D + col], __ldg(sc + row));
        default: {
            const uint8_t byte = base[row * ((D + 1) / 2) + col / 2];
            const int q = (col & 1) ? (byte & 15) : (byte >> 4);
            return __fmul_rn((float)(q - 8), __ldg(sc + row * ngroups + col / G));
        }
    }
}

// grid (n_pages + 1, B*H, parts), 256 threads.  Block (j, bh, part) covers the tokens from
// the end of page j-1 (0 for j = 0) to the end of page j (s_out for j = n_pages), in slices
// of part_tokens: the hole before page j becomes zeros, page j's rows are decoded.
template <bool VEC>
__global__ void __launch_bounds__(256) paged_gather_kernel(const skv_page_desc* __restrict__ table, int n_pages,
                                                          int D, int G, int64_t s_out, int64_t part_tokens,
                                                          float* __restrict__ k_out, float* __restrict__ v_out) {
    const int j = blockIdx.x, bh = blockIdx.y;
    __shared__ skv_page_desc s_pg;
    __shared__ long long s_lo;
    if (threadIdx.x == 0) {
        s_lo = j == 0 ? 0 : table[j - 1].start_token + table[j - 1].num_tokens;
        if (j < n_pages) {
            s_pg = table[j];
        } else {
            s_pg.start_token = s_out;
            s_pg.num_tokens = 0;
        }
    }
    __syncthreads();
    const int64_t lo = s_lo, pstart = s_pg.start_token, hi = pstart + s_pg.num_tokens;
    const int64_t a = lo + (int64_t)blockIdx.z * part_tokens;
    if (a >= hi) return;
    const int64_t b = min(hi, a + part_tokens);
    const int ngroups = D / G;
    // zeros for [a, min(b, pstart))
    const int64_t z1 = min(b, pstart);
    if (z1 > a) {
        const int64_t n4 = (z1 - a) * D / 4, o = ((int64_t)bh * s_out + a) * D;
        if (VEC) {
            const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int64_t i = threadIdx.x; i < n4; i += blockDim.x) {
                reinterpret_cast<float4*>(k_out + o)[i] = z;
                reinterpret_cast<float4*>(v_out + o)[i] = z;
            }
        } else {
            for (int64_t i = threadIdx.x; i < (z1 - a) * D; i += blockDim.x) {
                k_out[o + i] = 0.0f;
                v_out[o + i] = 0.0f;
            }
        }
    }
    // decoded rows for [max(a, pstart), b)
    const int64_t t0 = max(a, pstart);
    if (b <= t0) return;
    const int64_t row0 = (int64_t)bh * s_pg.row_stride + (t0 - pstart);
    const int64_t o = ((int64_t)bh * s_out + t0) * D;
    const int64_t n = (b - t0) * D;
    // 16-byte vector loads need 16-byte aligned payloads (4-byte scales); other pages decode
    // value by value
    const bool aligned = ((reinterpret_cast<uintptr_t>(s_pg.k) | reinterpret_cast<uintptr_t>(s_pg.v)) & 15) == 0 &&
                         ((reinterpret_cast<uintptr_t>(s_pg.scale_k) | reinterpret_cast<uintptr_t>(s_pg.scale_v)) & 3) == 0;
    if (VEC && aligned) {
        for (int64_t e = (int64_t)threadIdx.x * 8; e < n; e += (int64_t)blockDim.x * 8) {
            const int64_t r = e / D;
            const int col = (int)(e - r * D);
            float x[8];
            decode8(s_pg, false, row0 + r, col, D, ngroups, G, x);
            st8(k_out + o + e, x);
            decode8(s_pg, true, row0 + r, col, D, ngroups, G, x);
            st8(v_out + o + e, x);
        }
    } else {
        for (int64_t e = threadIdx.x; e < n; e += blockDim.x) {
            const int64_t r = e / D;
            const int col = (int)(e - r * D);
            k_out[o + e] = decode1(s_pg, false, row0 + r, col, D, ngroups, G);
            v_out[o + e] = decode1(s_pg, true, row0 + r, col, D, ngroups, G);
        }
    }
}

// One warp per (item, batch): items[i] = {table entry, row inside the page, head}.
__global__ void paged_clear_heads_kernel(const skv_page_desc* __restrict__ table, int n_pages,
                                         const int32_t* __restrict__ items, int64_t n_items, int B, int H, int D,
                                         int* __restrict__ bad) {
    const int lane = threadIdx.x & 31;
    const int64_t w = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (w >= n_items * B) return;
    const int64_t it = w / B;
    const int b = (int)(w % B);
    const int pos = items[3 * it], row = items[3 * it + 1], head = items[3 * it + 2];
    if (pos < 0 || pos >= n_pages || head < 0 || head >= H) {
        if (lane == 0) atomicExch(bad, 1);
        return;
    }
    const skv_page_desc pg = table[pos];
    if (row < 0 || row >= pg.num_tokens) {
        if (lane == 0) atomicExch(bad, 1);
        return;
    }
    const int64_t rb = paged_row_bytes(pg.precision, D);
    const int64_t r = (int64_t)(b * H + head) * pg.row_stride + row;
    const uint8_t fill = pg.precision == 3 ? 0x88 : 0x00;
    uint8_t* dk = static_cast<uint8_t*>(pg.k) + r * rb;
    uint8_t* dv = static_cast<uint8_t*>(pg.v) + r * rb;
    for (int64_t i = lane; i < rb; i += kWarp) {
        dk[i] = fill;
        dv[i] = fill;
    }
}

}  // namespace skv

using namespace skv;

extern "C" {

int skv_paged_write(const float* k, const float* v, int B, int H, int64_t T_src, int D, int int4_group_size,
                    const skv_page_write* writes, int n_writes, skv_page_desc* table, void* stream) {
    if (!k || !v || !writes) return fail(SKV_ERR_INVALID_ARGUMENT, "paged_write: null pointer");
    if (B <= 0 || H <= 0 || D <= 0 || T_src <= 0 || n_writes < 0)
        return fail(SKV_ERR_INVALID_ARGUMENT, "paged_write: bad size");
    if ((int64_t)B * H > (1 << 30)) return fail(SKV_ERR_TOO_LARGE, "paged_write: B*H above 2^30");
    if (n_writes == 0) return SKV_OK;
    const int G = int4_group(D, int4_group_size);
    if (int4_group_size <= 0) return fail(SKV_ERR_GROUP_SIZE, "paged_write: int4 group size must be positive");
    const int ngroups = D / G;
    const size_t smem = (size_t)kPagedWarps * ngroups * sizeof(unsigned);
    if (smem > 48 * 1024) return fail(SKV_ERR_UNSUPPORTED, "paged_write: %d int4 groups per row", ngroups);
    for (int i = 0; i < n_writes; ++i) {
        const skv_page_write& w = writes[i];
        const skv_page_desc& p = w.page;
        if (p.precision < 0 || p.precision > 3) return fail(SKV_ERR_INVALID_ARGUMENT, "paged_write: precision %d", p.precision);
        if (!p.k || !p.v || (p.precision >= 2 && (!p.scale_k || !p.scale_v)))
            return fail(SKV_ERR_INVALID_ARGUMENT, "paged_write: page %d has a null payload", i);
        if (w.rows <= 0 || w.dst_row < 0 || w.src_token < 0 || w.src_token + w.rows > T_src ||
            (int64_t)w.dst_row + w.rows > p.num_tokens || p.num_tokens > p.row_stride)
            return fail(SKV_ERR_SHAPE, "paged_write: write %d outside its page or source", i);
    }
    cudaStream_t st = as_stream(stream);
    const int BH = B * H;
    for (int base = 0; base < n_writes; base += kPagedManyWrites) {
        const int n = n_writes - base < kPagedManyWrites ? n_writes - base : kPagedManyWrites;
        int max_rows = 0;
        for (int i = 0; i < n; ++i) max_rows = writes[base + i].rows > max_rows ? writes[base + i].rows : max_rows;
        // vector path: whole rows per warp pass, int4 groups on aligned lane blocks
        const int V = D == 256 ? 8 : 4;
        bool vec = (D == 32 || D == 64 || D == 128 || D == 256) && G % V == 0;
        // 16-byte vectors: source rows and page payloads must start on 16-byte boundaries
        vec = vec && ((reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v)) & 15) == 0;
        for (int i = 0; i < n && vec; ++i) {
            const skv_page_desc& pg = writes[base + i].page;
            vec = ((reinterpret_cast<uintptr_t>(pg.k) | reinterpret_cast<uintptr_t>(pg.v)) & 15) == 0 &&
                  ((reinterpret_cast<uintptr_t>(pg.scale_k) | reinterpret_cast<uintptr_t>(pg.scale_v)) & 3) == 0;
        }
        int64_t gx;
        if (vec) {
            const int ppw = V == 8 ? 2 : 4;
            const int64_t passes = ((int64_t)max_rows * D + 32 * V - 1) / (32 * V);
            gx = (((passes + ppw - 1) / ppw) * BH + kPagedWarps - 1) / kPagedWarps;
        } else {
            gx = ((int64_t)max_rows * BH + kPagedWarps - 1) / kPagedWarps;
        }
        if (gx > 0x7fffffff) return fail(SKV_ERR_TOO_LARGE, "paged_write: grid too large");
        const dim3 grid((unsigned)gx, (unsigned)n);
        const int threads = kPagedWarps * kWarp;
        if (n <= kPagedFewWrites) {
            PagedWrites<kPagedFewWrites> ws;
            for (int i = 0; i < n; ++i) ws.w[i] = writes[base + i];
            if (!vec)
                paged_write_kernel<kPagedFewWrites><<<grid, threads, smem, st>>>(k, v, BH, T_src, D, G, ws, table);
            else if (V == 4)
                paged_write_vec_kernel<4, 4, kPagedFewWrites><<<grid, threads, 0, st>>>(k, v, BH, T_src, D, G, ws, table);
            else
                paged_write_vec_kernel<8, 2, kPagedFewWrites><<<grid, threads, 0, st>>>(k, v, BH, T_src, D, G, ws, table);
        } else {
            static PagedWrites<kPagedManyWrites> ws;   // 22.5 KB: kept off the host stack
            static std::mutex mu;
            std::lock_guard<std::mutex> lock(mu);
            for (int i = 0; i < n; ++i) ws.w[i] = writes[base + i];
            if (!vec)
                paged_write_kernel<kPagedManyWrites><<<grid, threads, smem, st>>>(k, v, BH, T_src, D, G, ws, table);
            else if (V == 4)
                paged_write_vec_kernel<4, 4, kPagedManyWrites><<<grid, threads, 0, st>>>(k, v, BH, T_src, D, G, ws,
                                                                                        table);
            else
                paged_write_vec_kernel<8, 2, kPagedManyWrites><<<grid, threads, 0, st>>>(k, v, BH, T_src, D, G, ws,
                                                                                        table);
        }
        const int rc = check_launch("paged_write");
        if (rc != SKV_OK) return rc;
    }
    return SKV_OK;
}

int skv_paged_gather(const skv_page_desc* table, int n_pages, int B, int H, int D, int int4_group_size,
                     int64_t s_out, int64_t max_span_tokens, float* k_out, float* v_out, void* stream) {
    if (!k_out || !v_out || (n_pages > 0 && !table)) return fail(SKV_ERR_INVALID_ARGUMENT, "paged_gather: null pointer");
    if (B <= 0 || H <= 0 || D <= 0 || n_pages < 0 || s_out < 0 || max_span_tokens < 0)
        return fail(SKV_ERR_INVALID_ARGUMENT, "paged_gather: bad size");
    if (int4_group_size <= 0) return fail(SKV_ERR_GROUP_SIZE, "paged_gather: int4 group size must be positive");
    if ((int64_t)B * H > 65535) return fail(SKV_ERR_TOO_LARGE, "paged_gather: B*H above 65535");
    if (s_out == 0 || max_span_tokens == 0) return SKV_OK;
    const int G = int4_group(D, int4_group_size);
    // about 8K output values per block and tensor; at most 65535 slices per page
    int64_t part = 8192 / D > 0 ? 8192 / D : 1;
    int64_t parts = (max_span_tokens + part - 1) / part;
    if (parts > 65535) {
        parts = 65535;
        part = (max_span_tokens + parts - 1) / parts;
    }
    const dim3 grid((unsigned)n_pages + 1, (unsigned)(B * H), (unsigned)parts);
    cudaStream_t st = as_stream(stream);
    const bool out_aligned = ((reinterpret_cast<uintptr_t>(k_out) | reinterpret_cast<uintptr_t>(v_out)) & 15) == 0;
    if (D % 8 == 0 && G % 8 == 0 && out_aligned)
        paged_gather_kernel<true><<<grid, 256, 0, st>>>(table, n_pages, D, G, s_out, part, k_out, v_out);
    else
        paged_gather_kernel<false><<<grid, 256, 0, st>>>(table, n_pages, D, G, s_out, part, k_out, v_out);
    return check_launch("paged_gather");
}

int skv_paged_clear_heads(const skv_page_desc* table, int n_pages, const int32_t* items, int64_t n_items, int B,
                          int H, int D, int* error_flag, void* stream) {
    if (!table || !items || !error_flag) return fail(SKV_ERR_INVALID_ARGUMENT, "paged_clear_heads: null pointer");
    if (B <= 0 || H <= 0 || D <= 0 || n_pages <= 0 || n_items < 0)
        return fail(SKV_ERR_INVALID_ARGUMENT, "paged_clear_heads: bad size");
    if (n_items == 0) return SKV_OK;
    const int64_t threads = n_items * B * kWarp;
    const int64_t blocks = (threads + 255) / 256;
    if (blocks > 0x7fffffff) return fail(SKV_ERR_TOO_LARGE, "paged_clear_heads: too many items");
    paged_clear_heads_kernel<<<(unsigned)blocks, 256, 0, as_stream(stream)>>>(table, n_pages, items, n_items, B, H, D,
                                                                             error_flag);
    return check_launch("paged_clear_heads");
}

}  // extern "C"
