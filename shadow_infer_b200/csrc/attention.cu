// Attention read from the packed cache, on the sm_100a tensor cores.
//
// Oracle: PackedKVCache.unpack() (shadowinfer/shadowkv/packed_kv_cache.py:535-577) followed by
// the dense, non-causal attention of SimpleDiffusionLLM._compute_block
// (shadowinfer/models/simple_diffusion_llm.py:165-169): O = softmax(Q K^T / sqrt(D)) V with
// evicted (t,h) entries present as ZERO rows of K and V (logit 0, no value).
//
// skv_head_index       -- per head, the stored entries of the cache grouped by precision (token
//                         order inside a group): the KV row list the attention walks.
// skv_packed_attention -- two launches on the caller's stream:
//   1. stage_tiles_kernel (skv_stage_kv_tiles), one CTA per (128-row KV tile, head, batch):
//      gathers the tile's rows from the fp32/fp16/int8/int4 buckets and dequantises them ONCE
//      into fp16 K and V tiles in exactly the byte layout the tensor cores read (128B-swizzled
//      atoms of 128 rows x 64 values), K and V with RNE (fp32 -> fp16) of the value the reference
//      dequantises (q * scale for int8 / int4, computed in fp32 as the reference does).  Beside
//      them, per KV head, the lo part RNE(k - RNE(k)) of the 16 channels of largest max |K|
//      (channel-selective lo, see kLoCh), unless the tile is all fp16 entries and so exact.
//      Evicted entries are not staged.  Every query tile of the head reuses the staged tiles
//      (from L2), so the packed bytes are read and converted once per head instead of once per
//      query tile.
//   2. packed_attention_kernel (skv_attend_kv_tiles): persistent, one CTA per SM, launched
//      cooperatively.  A work unit is 256 queries (two 128-row tiles) of one head.  Whole units
//      go round-robin over the CTAs (the units in flight share one or two heads' tiles in L2);
//      the last one to two rounds are split evenly by KV steps (a unit cut between two CTAs is
//      merged through a partial (O, max, sum) in scratch).  Per CTA:
//      warps 0-7  softmax, two groups of four: group t owns query tile t, thread i of the group
//                 owns query row i = TMEM lane i.  Reads S_t from TMEM, keeps the running max
//                 and sum (lazy rescale of O_t when the max grows by more than 2^8), and writes
//                 P_t (fp16) back into TMEM over the first half of S_t's columns; at the end of
//                 a unit, normalises O_t and stores it.
//      warp 8     loader: Q tiles by TMA (128B swizzle, no multicast), the staged K (+ lo) and
//                 V tiles by bulk asynchronous copies into two-stage rings, and the queries'
//                 selected channels Q_c gathered from the Q tiles.
//      warp 9     MMA issuer (tcgen05.mma kind::f16, M=128, fp32 accumulate):
//                 S_t = Q_t K_j^T (+ Q_c,t K_lo,j^T over the selected channels; both operands in
//                 shared memory) and O_t += P_t V_j (P read from TMEM), interleaved PV_0(j),
//                 S_0(j+1), PV_1(j), S_1(j+1) so that the tensor cores work on one query tile
//                 while the other tile's softmax runs.  One thread issues every MMA: the issue
//                 of a tcgen05.mma costs about as long as its execution at N = 128, so two issuers
//                 (one per group) interleave their tiles' MMAs in the pipe, and a hand-over
//                 between them leaves the pipe idle for the hand-over's latency (measured).
//      TMEM: S_0 | S_1 | O_0 | O_1 (128 + 128 + D + D columns).
// Evicted entries never enter a tile: their contribution (count * 2^(0 - m)) is added to the
// softmax denominator analytically.  Every mbarrier wait is bounded; a timeout sets the error
// word and all roles drain to the final barrier before TMEM is released.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <math.h>
#include <string.h>

#include <mutex>

#include "skv_common.cuh"
#include "sm100_ptx.cuh"

namespace skv {
using namespace sm100;

constexpr int kBM = 128;          // queries per tile (two tiles per CTA)
constexpr int kBN = 128;          // KV rows per tile
constexpr int kSoftmaxWarps = 8;
constexpr int kLoadWarp = 8;
constexpr int kMmaWarp = 9;
constexpr int kAttnThreads = 10 * 32;
constexpr int kStageThreads = 256;
constexpr uint32_t kTmemCols = 512;
constexpr float kRescaleThreshold = 8.0f;   // log2 units

enum AttnError { kErrNone = 0, kErrKFull = 1, kErrKEmpty = 2, kErrSFull = 3, kErrPFull = 4, kErrOFull = 5,
                 kErrDrain = 6, kErrQFull = 7, kErrVFull = 8, kErrVEmpty = 9, kErrCopy = 10, kErrQEmpty = 11,
                 kErrOEmpty = 12, kErrPartial = 13, kErrSchedule = 14, kErrTurn = 15 };

// Bytes of one staged K (or V) tile: D/64 swizzle atoms of 128 rows x 128 bytes.
__host__ __device__ constexpr int staged_tile_bytes(int D) { return (D / 64) * kBN * 128; }

constexpr int kLoCh = 16;                       // channels of K with a lo part: one MMA K-step of fp16
constexpr int kLoTile = kBN * kLoCh * 2;        // their lo tile: 128 rows x 32 bytes (32-byte swizzle)

constexpr int kMaxHeads = 256;     // heads per launch (the schedule keeps a per-head prefix in smem)
constexpr int kMaxPartners = 8;    // CTAs that can hold later parts of one unit (merged by its first part)
// bytes of the schedule's shared state (SchedSmem: 48 bytes of fields, the two prefixes)
constexpr int kSchedSmemBytes = (48 + (kMaxHeads + 1) * 4 + (kMaxHeads + 1) * 2 + 15) / 16 * 16;
constexpr int kUnitRows = 2 * kBM;  // queries per work unit

template <int D, bool PEERS = false>
struct AttnLayout {
    static constexpr int NA = D / 64;                   // 128-byte swizzle atoms per row
    static constexpr int kTile = staged_tile_bytes(D);  // one 128-row tile (Q, K or V)
    static constexpr int kQ = 0;                        // two query tiles
    static constexpr int kK = kQ + 2 * kTile;           // two K stages
    static constexpr int kV = kK + 2 * kTile;           // two V stages
    static constexpr int kQc = kV + 2 * kTile;          // two tiles of the queries' selected channels (32B swizzle)
    static constexpr int kKc = kQc + 2 * kLoTile;       // two stages of K lo of the selected channels
    static constexpr int kBar = kKc + 2 * kLoTile;
    static constexpr int kNumBars = 24;
    static constexpr int kSch = kBar + kNumBars * 8;    // SchedSmem (defined below)
    // PEERS: per softmax warp, kOutRows output rows staged for the bulk stores into every rank's buffer
    static constexpr int kOut = (kSch + kSchedSmemBytes + 127) / 128 * 128;
    static constexpr int kOutRows = 4;
    static constexpr int kMisc = kOut + (PEERS ? kSoftmaxWarps * kOutRows * D * 4 : 0);
    static constexpr int kTmemSlot = kMisc + 16;
    static constexpr int kBytes = kTmemSlot + 16;
    // + slack to align the base to 1024 B; at least 120 KB so that one CTA occupies an SM and
    // its 512-column TMEM allocation never waits for another CTA's
    static constexpr int kAlloc = (kBytes + 1024) > 120 * 1024 ? (kBytes + 1024) : 120 * 1024;
    static_assert(kAlloc <= 227 * 1024, "attention shared memory beyond the per-CTA limit");
};

struct AttnParams {
    const __half* q;           // [B, H, S_q, D]
    float* out;                // [B, H, S_q, D]
    Buckets bk;
    const int32_t* rows;       // [H_kv, S_kv] slot values of the stored entries, grouped by precision
    const int32_t* counts;     // [H_kv, 5]: stored entries per precision, evicted entries
    const float* k_new;        // [B, H_kv, S_new, D] dense rows attended after the packed ones (or NULL)
    const float* v_new;
    uint8_t* stage;            // [B, H_kv, ntmax, 2 (K, V), staged_tile_bytes(D)]
    float* part_o;             // [slots, kUnitRows, D]: unnormalised O of a unit's second part
    float2* part_ml;           // [slots, kUnitRows]: its (reference max, sum) per query row
    int* part_flag;            // [slots]: softmax warps that have published their rows
    int B, H, S_q, S_kv, G, ntmax, QP, slots;
    int H_kv, rep, S_new;      // query head h reads KV head h / rep (grouped-query attention)
    // outputs written straight into n_peers buffers [B, H_out, S_q, D] (this rank's heads at
    // head_off; peers' memory over NVLink), or into `out` [B, H, S_q, D] when n_peers == 0
    float* const* peers;
    int n_peers, head_off, H_out;
    float scale_log2;          // softmax scale * log2(e)
    int* err;
    int klo;                   // 1: the head's kLoCh largest channels of K also contribute their lo part
    int one_tile;              // 1: the single-query-tile kernel (units of 128 queries); 0: two tiles (256)
    int pair;                  // 1: the CTA-pair kernel (units of 256 queries over two CTAs, head_dim 128)
    int out_half;              // 1: `out` and every peer buffer hold fp16 (two-tile kernel only)
    int emu;                   // two-tile kernel: a quarter of the exponentials on the FMA pipe
    unsigned* chmax;           // [H_kv, D] max |K| per channel (float bits), channel selection input
    int* sel;                  // [H_kv, kLoCh] the selected channels, ascending
};

__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ float fmax3(float a, float b, float c) {
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}

// Max of N floats (bit patterns) as a tree of 3-input maxes: depth log3(N) instead of a chain,
// the max's latency rather than its instruction count bounds the softmax's first pass.
template <int N>
__device__ __forceinline__ float row_max(const uint32_t* v) {
    float a[(N + 2) / 3];
#pragma unroll
    for (int i = 0; i < N / 3; ++i)
        a[i] = fmax3(__uint_as_float(v[3 * i]), __uint_as_float(v[3 * i + 1]), __uint_as_float(v[3 * i + 2]));
    if constexpr (N % 3 == 1) a[N / 3] = __uint_as_float(v[N - 1]);
    if constexpr (N % 3 == 2) a[N / 3] = fmaxf(__uint_as_float(v[N - 2]), __uint_as_float(v[N - 1]));
    constexpr int M = (N + 2) / 3;
    if constexpr (M == 1) {
        return a[0];
    } else {
        uint32_t b[M];
#pragma unroll
        for (int i = 0; i < M; ++i) b[i] = __float_as_uint(a[i]);
        return row_max<M>(b);
    }
}

__device__ __forceinline__ uint32_t half2_bits(__half2 h) {
    uint32_t u;
    memcpy(&u, &h, 4);
    return u;
}

// Warp-uniform bounded wait: every lane polls, and the warp fails together if any lane gave
// up, so .sync.aligned tcgen05 instructions that follow stay convergent.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, int* err, int code) {
    const bool ok = mbar_wait_spin(bar, parity, err, code);
    return __all_sync(0xffffffffu, ok);
}

// Channel-selective lo part of K.  fp16 K is off by up to 2^-11 of every element; a few channels
// of much larger magnitude than the rest (channel outliers of K) make that the dominant error of
// the scores.  Per KV head the kLoCh channels of largest max |K| get lo = RNE(k - RNE(k)) staged
// in a small tile of their own, and one extra MMA (K = kLoCh) adds Q[:, sel] K_lo^T to the scores,
// so these channels enter with ~22 bits and the rest with fp16's 11 (kLoCh, kLoTile above).
// Staged tiles of (batch b, KV head h, tile j), contiguous: K (fp16), V (fp16), K lo of the
// selected channels.
__host__ __device__ constexpr int staged_set_bytes(int D) { return 2 * staged_tile_bytes(D) + kLoTile; }
constexpr int kSetKHi = 0, kSetV = 1;           // in units of staged_tile_bytes; the lo tile follows V
__device__ __forceinline__ int64_t staged_offset(const AttnParams& p, int b, int h, int j, int D) {
    return (((int64_t)b * p.H_kv + h) * p.ntmax + j) * staged_set_bytes(D);
}

// Byte offset of 16-byte chunk `chunk` (0..1) of row `row` of a 32-byte-swizzled K-major tile
// (rows 32 bytes apart; the chunk index is XORed with bit 2 of the row, the pattern of the
// SWIZZLE_32B shared-memory descriptor and tensor map).
__device__ __forceinline__ uint32_t sw32_offset(int row, int chunk) {
    return (uint32_t)(row * 32 + ((chunk ^ ((row >> 2) & 1)) << 4));
}

// Rows [c0, c1) of a head's row list are its fp16 entries (the list holds fp32, fp16, int8,
// int4 entries in that order, then the dense new rows).  A tile inside them is exact in fp16.
struct HeadRows {
    int f16_begin, f16_end, n_rows;
    int klo;
    __device__ __forceinline__ void load(const AttnParams& p, int h);
    __device__ __forceinline__ bool exact(int j) const {
        const int lo = j * kBN, hi = min(lo + kBN, n_rows);
        return !klo || (lo >= f16_begin && hi <= f16_end);
    }
};
__device__ __forceinline__ void HeadRows::load(const AttnParams& p, int h) {
    const int* c = p.counts + (int64_t)(h / p.rep) * 5;
    const int c0 = __ldg(c), c1 = __ldg(c + 1), c2 = __ldg(c + 2), c3 = __ldg(c + 3);
    f16_begin = c0;
    f16_end = c0 + c1;
    n_rows = c0 + c1 + c2 + c3 + p.S_new;
    klo = p.klo;
}

// ------------------------------------------------------------------------------ staging
// Eight int4 codes (one word, high nibble first per byte) times a group scale, in fp32 exactly
// as the reference dequantises ((nibble - 8) * scale).
__device__ __forceinline__ void int4x8_to_f32(uint32_t w, float s, float (&v)[8]) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint32_t byte = (w >> (8 * i)) & 0xFFu;
        v[2 * i] = __fmul_rn(__int_as_float(0x4B000000 | (byte >> 4)) - 8388616.0f, s);
        v[2 * i + 1] = __fmul_rn(__int_as_float(0x4B000000 | (byte & 0xF)) - 8388616.0f, s);
    }
}

// Eight int8 codes times the row scale, in fp32 exactly as the reference dequantises
// (q * scale).  (q ^ 0x80) | 0x4B000000 is 2^23 + q + 128.
__device__ __forceinline__ void int8x8_to_f32(uint32_t w0, uint32_t w1, float s, float (&v)[8]) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        v[i] = __fmul_rn(__int_as_float(0x4B000000 | (((w0 >> (8 * i)) & 0xFFu) ^ 0x80u)) - 8388736.0f, s);
        v[4 + i] = __fmul_rn(__int_as_float(0x4B000000 | (((w1 >> (8 * i)) & 0xFFu) ^ 0x80u)) - 8388736.0f, s);
    }
}

__device__ __forceinline__ uint4 f32x8_to_half(const float (&v)[8]) {
    uint4 r;
    r.x = half2_bits(__floats2half2_rn(v[0], v[1]));
    r.y = half2_bits(__floats2half2_rn(v[2], v[3]));
    r.z = half2_bits(__floats2half2_rn(v[4], v[5]));
    r.w = half2_bits(__floats2half2_rn(v[6], v[7]));
    return r;
}

// hi = RNE(v), lo = RNE(v - hi) for eight fp32 values (v - hi is exact in fp32).  A K element
// in fp16 alone is off by up to 2^-11 of itself, and channel outliers of K (a few channels ten
// times larger than the rest) make that the dominant error of the attention; hi + lo keeps
// the contraction within ~2^-22.
__device__ __forceinline__ void f32x8_split(const float (&v)[8], uint4& hi, uint4& lo) {
    uint32_t h[4], l[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const __half2 hh = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
        const float2 hf = __half22float2(hh);
        h[i] = half2_bits(hh);
        l[i] = half2_bits(__floats2half2_rn(v[2 * i] - hf.x, v[2 * i + 1] - hf.y));
    }
    hi = make_uint4(h[0], h[1], h[2], h[3]);
    lo = make_uint4(l[0], l[1], l[2], l[3]);
}

__device__ __forceinline__ void f32x8_load(const float* src, float (&v)[8]) {
    const float4 a = __ldg(reinterpret_cast<const float4*>(src));
    const float4 b = __ldg(reinterpret_cast<const float4*>(src) + 1);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

// Raw packed bytes of one lane's share of one K row and one V row: chunk `l8` (8 values)
// of each 64-value atom, plus the row/group scales.  Loaded for several rows before any is
// converted, so each lane keeps several memory requests in flight.  fp32 rows (packed fp32
// entries and the dense new rows) carry V converted at load and a pointer to their K row,
// which is read when the row is stored (it is split into hi + lo there).
template <int NA>
struct RawRow {
    uint4 k[NA], v[NA];         // fp16, int8 8 bytes, int4 4 bytes (unused for K of fp32 rows)
    float sk[NA], sv[NA];
    const float* kf;            // fp32 rows: K row
    int code;                   // 0 fp32 row, 1..3 packed fp16 / int8 / int4, -1 padding row
};

template <int D, bool WANT_V = true>
__device__ __forceinline__ void load_raw_row(const AttnParams& p, int b, int32_t e, int l8, RawRow<D / 64>& r) {
    constexpr int NA = D / 64;
    r.code = e < 0 ? -1 : slot_code(e);
    if (e < 0) return;
    const int64_t row = (int64_t)slot_pos(e) * p.B + b;
    const skv_bucket& bb = p.bk.b[r.code];
    if (r.code == 0) r.kf = reinterpret_cast<const float*>(bb.k) + row * D;
#pragma unroll
    for (int a = 0; a < NA; ++a) {
        const int d0 = a * 64 + l8 * 8;
        if (r.code == 0) {
            // rare: V converted at once (RNE), K read again when stored
            if (WANT_V) {
                float x[8];
                f32x8_load(reinterpret_cast<const float*>(bb.v) + row * D + d0, x);
                r.v[a] = f32x8_to_half(x);
            }
        } else if (r.code == 1) {
            r.k[a] = __ldg(reinterpret_cast<const uint4*>(reinterpret_cast<const __half*>(bb.k) + row * D + d0));
            if (WANT_V)
                r.v[a] = __ldg(reinterpret_cast<const uint4*>(reinterpret_cast<const __half*>(bb.v) + row * D + d0));
        } else if (r.code == 2) {
            const uint2 wk = __ldg(reinterpret_cast<const uint2*>(reinterpret_cast<const int8_t*>(bb.k) + row * D + d0));
            r.k[a] = make_uint4(wk.x, wk.y, 0, 0);
            if (WANT_V) {
                const uint2 wv = __ldg(reinterpret_cast<const uint2*>(reinterpret_cast<const int8_t*>(bb.v) + row * D + d0));
                r.v[a] = make_uint4(wv.x, wv.y, 0, 0);
            }
            if (a == 0) {
                r.sk[0] = __ldg(bb.scale_k + row);
                if (WANT_V) r.sv[0] = __ldg(bb.scale_v + row);
            }
        } else {
            const int64_t off = (int64_t)slot_pos(e) * ((int64_t)p.B * D / 2) + (int64_t)b * (D / 2) + d0 / 2;
            r.k[a].x = __ldg(reinterpret_cast<const uint32_t*>(reinterpret_cast<const uint8_t*>(bb.k) + off));
            const int NG = D / p.G;
            const int g = d0 / p.G;
            r.sk[a] = __ldg(bb.scale_k + row * NG + g);
            if (WANT_V) {
                r.v[a].x = __ldg(reinterpret_cast<const uint32_t*>(reinterpret_cast<const uint8_t*>(bb.v) + off));
                r.sv[a] = __ldg(bb.scale_v + row * NG + g);
            }
        }
    }
}

// One lane's share of dense fp32 row r of (b, KV head h) of k_new / v_new: V converted to fp16,
// K kept as a pointer (split when stored).
template <int D, bool WANT_V = true>
__device__ __forceinline__ void load_dense_row(const AttnParams& p, int b, int h, int r, int l8, RawRow<D / 64>& raw) {
    constexpr int NA = D / 64;
    raw.code = 0;
    const int64_t row = (((int64_t)b * p.H_kv + h) * p.S_new + r) * D;
    raw.kf = p.k_new + row;
    if (!WANT_V) return;
#pragma unroll
    for (int a = 0; a < NA; ++a) {
        float x[8];
        f32x8_load(p.v_new + row + a * 64 + l8 * 8, x);
        raw.v[a] = f32x8_to_half(x);
    }
}

// The eight fp32 K values of atom `a` of one lane's share of a row (zeros for a padding row).
template <int D>
__device__ __forceinline__ void raw_k_f32(const RawRow<D / 64>& raw, int a, int l8, float (&x)[8]) {
    if (raw.code == 0) {
        f32x8_load(raw.kf + a * 64 + l8 * 8, x);
    } else if (raw.code == 1) {
        const uint32_t w[4] = {raw.k[a].x, raw.k[a].y, raw.k[a].z, raw.k[a].w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            __half2 h2;
            memcpy(&h2, &w[i], 4);
            const float2 f = __half22float2(h2);
            x[2 * i] = f.x;
            x[2 * i + 1] = f.y;
        }
    } else if (raw.code == 2) {
        int8x8_to_f32(raw.k[a].x, raw.k[a].y, raw.sk[0], x);
    } else if (raw.code == 3) {
        int4x8_to_f32(raw.k[a].x, raw.sk[a], x);
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) x[i] = 0.0f;
    }
}

// Converts one lane's share of a K and a V row to fp16 and stores it, 128B-swizzled, at row `r`
// of the staged tiles (zeros for a padding row); with `want_lo`, the lo parts of the selected
// channels that fall in this lane's chunks go to the lo tile (bit i of lo_bits[a]: selected
// channel i lies in chunk a; its position inside the chunk is lo_pos[i]).
template <int D>
__device__ __forceinline__ void store_row(const RawRow<D / 64>& raw, int r, int l8, uint8_t* ktile, uint8_t* vtile,
                                          uint8_t* lotile, bool want_lo, const uint32_t (&lo_bits)[D / 64],
                                          const int8_t* lo_pos) {
    constexpr int NA = D / 64;
#pragma unroll
    for (int a = 0; a < NA; ++a) {
        float x[8];
        raw_k_f32<D>(raw, a, l8, x);
        uint4 hv = make_uint4(0, 0, 0, 0);
        if (raw.code == 0 || raw.code == 1) {
            hv = raw.v[a];
        } else if (raw.code == 2) {
            float y[8];
            int8x8_to_f32(raw.v[a].x, raw.v[a].y, raw.sv[0], y);
            hv = f32x8_to_half(y);
        } else if (raw.code == 3) {
            float y[8];
            int4x8_to_f32(raw.v[a].x, raw.sv[a], y);
            hv = f32x8_to_half(y);
        }
        const uint4 hk = raw.code == 1 ? raw.k[a] : f32x8_to_half(x);
        const int off = a * kBN * 128 + sw128_offset(r, l8);
        *reinterpret_cast<uint4*>(ktile + off) = hk;
        *reinterpret_cast<uint4*>(vtile + off) = hv;
        if (want_lo) {
            for (uint32_t bits = lo_bits[a]; bits; bits &= bits - 1) {
                const int i = __ffs(bits) - 1;
                const float v = x[lo_pos[i]];
                const __half lo = __float2half_rn(v - __half2float(__float2half_rn(v)));
                *reinterpret_cast<__half*>(lotile + sw32_offset(r, i >> 3) + (i & 7) * 2) = lo;
            }
        }
    }
}

// The selected channels of KV head h (shared memory) and this lane's share of them: bit i of
// lo_bits[a] is set when selected channel i lies in chunk (a, l8); lo_pos[i] is its position in
// the chunk.
template <int D>
__device__ __forceinline__ void lo_share(const AttnParams& p, int h, int l8, int* s_sel, uint32_t (&lo_bits)[D / 64],
                                         int8_t* s_pos) {
    if (threadIdx.x < kLoCh) {
        const int c = p.klo ? __ldg(p.sel + (int64_t)h * kLoCh + threadIdx.x) : 0;
        s_sel[threadIdx.x] = c;
        s_pos[threadIdx.x] = (int8_t)(c & 7);
    }
    __syncthreads();
#pragma unroll
    for (int a = 0; a < D / 64; ++a) {
        uint32_t bits = 0;
#pragma unroll
        for (int i = 0; i < kLoCh; ++i)
            if ((s_sel[i] >> 3) == a * 8 + l8) bits |= 1u << i;
        lo_bits[a] = bits;
    }
}

// One CTA per (KV tile j, KV head h, batch b); tiles past the head's rows exit at once.  A
// head's rows are its stored packed entries, then the S_new dense rows of k_new / v_new.
// Eight lanes per row (one 16-byte chunk of each atom per lane), 32 rows per pass, 4 passes.
// The row-list entries are fetched together with the head's counts (entries past the stored
// rows are discarded afterwards), so a CTA waits for two memory round trips, not three.
template <int D>
__global__ void __launch_bounds__(kStageThreads, 2) stage_tiles_kernel(AttnParams p) {
    constexpr int NA = D / 64;
    constexpr int kRowsPerPass = kStageThreads / 8;
    constexpr int kPasses = kBN / kRowsPerPass;
    __shared__ int s_sel[kLoCh];
    __shared__ int8_t s_pos[kLoCh];
    const int j = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    const int rsub = threadIdx.x >> 3, l8 = threadIdx.x & 7;
    const int32_t* hrows = p.rows + (int64_t)h * p.S_kv;
    int32_t e[kPasses];
#pragma unroll
    for (int i = 0; i < kPasses; ++i) {
        const int idx = j * kBN + i * kRowsPerPass + rsub;
        e[i] = idx < p.S_kv ? __ldg(hrows + idx) : -1;
    }
    HeadRows hr;
    hr.load(p, h);
    const int n_stored = hr.n_rows - p.S_new;
    if (j * kBN >= hr.n_rows) return;
    const bool want_lo = !hr.exact(j);
    uint32_t lo_bits[NA];
    lo_share<D>(p, h, l8, s_sel, lo_bits, s_pos);
    const int TB = staged_tile_bytes(D);
    uint8_t* ktile = p.stage + staged_offset(p, b, h, j, D);
    uint8_t* vtile = ktile + TB;
    uint8_t* lotile = ktile + 2 * TB;
    RawRow<NA> raw[kPasses];
#pragma unroll
    for (int i = 0; i < kPasses; ++i) {
        const int idx = j * kBN + i * kRowsPerPass + rsub;
        if (idx >= n_stored && idx < hr.n_rows)
            load_dense_row<D>(p, b, h, idx - n_stored, l8, raw[i]);
        else
            load_raw_row<D>(p, b, idx < n_stored ? e[i] : -1, l8, raw[i]);
    }
#pragma unroll
    for (int i = 0; i < kPasses; ++i)
        store_row<D>(raw[i], i * kRowsPerPass + rsub, l8, ktile, vtile, lotile, want_lo, lo_bits, s_pos);
}

// Max |K| per channel of each KV head over all its rows and batches (float bits, atomicMax on
// non-negative floats orders like the values): the input of the channel selection.  Same grid
// and row mapping as the staging; `chmax` is cleared before the launch.
template <int D>
__global__ void __launch_bounds__(kStageThreads, 2) chan_max_kernel(AttnParams p) {
    constexpr int NA = D / 64;
    constexpr int kRowsPerPass = kStageThreads / 8;
    constexpr int kPasses = kBN / kRowsPerPass;
    __shared__ unsigned s_max[D];
    const int j = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    const int rsub = threadIdx.x >> 3, l8 = threadIdx.x & 7;
    HeadRows hr;
    hr.load(p, h);
    const int n_stored = hr.n_rows - p.S_new;
    if (j * kBN >= hr.n_rows) return;
    for (int d = threadIdx.x; d < D; d += kStageThreads) s_max[d] = 0u;
    __syncthreads();
    const int32_t* hrows = p.rows + (int64_t)h * p.S_kv;
    float m[NA][8];
#pragma unroll
    for (int a = 0; a < NA; ++a)
#pragma unroll
        for (int i = 0; i < 8; ++i) m[a][i] = 0.0f;
    // all rows' K bytes in flight before any is reduced (V is not read)
    int32_t e[kPasses];
#pragma unroll
    for (int i = 0; i < kPasses; ++i) {
        const int idx = j * kBN + i * kRowsPerPass + rsub;
        e[i] = idx < n_stored ? __ldg(hrows + idx) : -1;
    }
    RawRow<NA> raw[kPasses];
#pragma unroll
    for (int i = 0; i < kPasses; ++i) {
        const int idx = j * kBN + i * kRowsPerPass + rsub;
        if (idx >= n_stored && idx < hr.n_rows)
            load_dense_row<D, false>(p, b, h, idx - n_stored, l8, raw[i]);
        else
            load_raw_row<D, false>(p, b, e[i], l8, raw[i]);
    }
#pragma unroll
    for (int i = 0; i < kPasses; ++i) {
#pragma unroll
        for (int a = 0; a < NA; ++a) {
            float x[8];
            raw_k_f32<D>(raw[i], a, l8, x);
#pragma unroll
            for (int t = 0; t < 8; ++t) m[a][t] = fmaxf(m[a][t], fabsf(x[t]));
        }
    }
#pragma unroll
    for (int a = 0; a < NA; ++a)
#pragma unroll
        for (int t = 0; t < 8; ++t)
            if (m[a][t] > 0.0f) atomicMax(&s_max[a * 64 + l8 * 8 + t], __float_as_uint(m[a][t]));
    __syncthreads();
    for (int d = threadIdx.x; d < D; d += kStageThreads)
        if (s_max[d]) atomicMax(p.chmax + (int64_t)h * D + d, s_max[d]);
}

// Per KV head, the kLoCh channels of largest max |K| (ties: lower channel first), written in
// ascending channel order.  One block of D threads per head.
template <int D>
__global__ void __launch_bounds__(D) chan_select_kernel(AttnParams p) {
    __shared__ unsigned s_v[D];
    __shared__ int s_flag[D];
    const int h = blockIdx.x, d = threadIdx.x;
    const unsigned v = p.chmax[(int64_t)h * D + d];
    s_v[d] = v;
    __syncthreads();
    int rank = 0;
    for (int e = 0; e < D; ++e) {
        const unsigned w = s_v[e];
        rank += (w > v || (w == v && e < d)) ? 1 : 0;
    }
    const bool chosen = rank < kLoCh;
    s_flag[d] = chosen ? 1 : 0;
    __syncthreads();
    if (chosen) {
        int pos = 0;
        for (int e = 0; e < d; ++e) pos += s_flag[e];
        p.sel[(int64_t)h * kLoCh + pos] = d;
    }
}

// ------------------------------------------------------------------------------ attention
// Work schedule.  A unit is (batch b, head h, query pair qp): 256 queries against the head's
// nt_h staged KV tiles, one step per tile.  Units are ordered (b, h, qp) with qp fastest and
// their steps laid end to end; CTA c of the G working CTAs takes the contiguous step range
// [c*T/G, (c+1)*T/G).  G <= T / max(nt_h), so every range holds at least one whole unit's
// worth of steps and a unit is cut at most once: its first part (steps [0, k)) is the last
// segment of CTA c, its second part (steps [k, nt)) the first segment of CTA c+1.
struct Segment {
    int b, h, qp, j0, j1, nt;
};

// The schedule's shared state, written by one thread before the CTA's first barrier: per-head
// prefixes hp[h] = KV tiles of heads before h and hn[h] = heads before h that have any tile, and
// the split of the work over the grid (below).  Each thread keeps only its cursor in registers.
struct SchedSmem {
    long long per_batch;       // steps of one batch entry: QP * hp[H]
    long long P0, T_sk;        // first step and step count of the stream-K tail
    int H, QP, G, G_sk;        // heads, query blocks per head, CTAs, CTAs sharing the tail (0: none)
    int unit_end;              // data-parallel units: [0, unit_end)
    int ntm;                   // largest tile count of a head
    int hp[kMaxHeads + 1];
    uint16_t hn[kMaxHeads + 1];
};

// Work of one CTA.  Units (batch, head, query block) are ordered batch-major, then head, then
// query block; a unit is nt steps (one per KV tile of its head).
//  * Data-parallel rounds: CTA c takes whole units c, c + G, c + 2G, ... for the first
//    `rounds` x G units, so the G units in flight at any time are consecutive -- they share one
//    or two heads' staged K/V, which stays in L2 instead of every CTA streaming its own head.
//  * Stream-K tail (the last one to two rounds of units): their steps are split contiguously,
//    CTA c taking steps [bound(c), bound(c + 1)); a unit cut at a CTA boundary has its first part
//    in the lower CTA, which merges the later parts published by the CTAs above it.  G_sk keeps at
//    least ceil(max_nt / kMaxPartners) steps per CTA, so a unit spans at most kMaxPartners + 1.
static_assert(sizeof(SchedSmem) <= kSchedSmemBytes, "schedule state beyond its shared-memory slot");

struct Schedule {
    const SchedSmem* c;
    int unit;                  // next data-parallel unit of this CTA (steps of G)
    long long pos, end;        // this CTA's tail steps

    __device__ long long bound(long long cta) const { return c->P0 + cta * c->T_sk / c->G_sk; }

    // (b, h, qp, nt) of unit u and its first step
    __device__ static long long unit_start(const SchedSmem* c, long long u, int& b, int& h, int& qp, int& nt) {
        const long long upb = (long long)c->QP * c->hn[c->H];
        const long long bb = u / upb;
        const long long r = u - bb * upb;
        const int k = (int)(r / c->QP);
        // largest h with hn[h] <= k: the k-th head that has tiles
        int lo = 0, hi = c->H - 1;
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (c->hn[mid] <= k) lo = mid;
            else hi = mid - 1;
        }
        b = (int)bb;
        h = lo;
        qp = (int)(r - (long long)k * c->QP);
        nt = c->hp[lo + 1] - c->hp[lo];
        return bb * c->per_batch + (long long)c->QP * c->hp[lo] + (long long)qp * nt;
    }

    // one thread: head prefixes and the split (before the CTA's first barrier)
    __device__ static void setup(SchedSmem* c, const AttnParams& p) {
        int acc = 0, heads = 0, ntm = 0;    // acc below 2^31: H * ntmax is checked on the host
        for (int hh = 0; hh < p.H; ++hh) {
            const int* cn = p.counts + (int64_t)(hh / p.rep) * 5;
            const int n = (cn[0] + cn[1] + cn[2] + cn[3] + p.S_new + kBN - 1) / kBN;
            c->hp[hh] = acc;
            c->hn[hh] = (uint16_t)heads;
            acc += n;
            heads += n > 0;
            ntm = max(ntm, n);
        }
        c->hp[p.H] = acc;
        c->hn[p.H] = (uint16_t)heads;
        c->ntm = ntm;
        c->H = p.H;
        c->QP = p.QP;
        c->G = (int)gridDim.x;
        c->per_batch = (long long)p.QP * acc;
        const long long T = c->per_batch * p.B;
        const long long U = (long long)p.B * p.QP * heads;     // below 2^31: B * H * S_q is checked
        const long long rounds = U / c->G >= 2 ? U / c->G - 1 : 0;
        c->unit_end = (int)(rounds * c->G);
        c->P0 = T;
        if (c->unit_end < U) {
            int b, h, qp, nt;
            c->P0 = unit_start(c, c->unit_end, b, h, qp, nt);
        }
        c->T_sk = T - c->P0;
        c->G_sk = 0;
        if (c->T_sk > 0) {
            const long long cap = max(1ll, c->T_sk / ((ntm + kMaxPartners - 1) / kMaxPartners));
            c->G_sk = (int)min((long long)c->G, cap);
        }
    }

    __device__ void init(const SchedSmem* c_) {
        c = c_;
        unit = blockIdx.x;
        pos = end = 0;
        if ((int)blockIdx.x < c->G_sk) {
            pos = bound(blockIdx.x);
            end = bound((long long)blockIdx.x + 1);
        }
    }

    // out of line (once per segment): its registers stay out of the roles' loops
    __device__ __noinline__ bool next(Segment& s) {
        if (unit < c->unit_end) {
            unit_start(c, unit, s.b, s.h, s.qp, s.nt);
            s.j0 = 0;
            s.j1 = s.nt;
            unit += c->G;
            return true;
        }
        if (pos >= end) return false;
        const long long bb = pos / c->per_batch;
        const long long r = pos - bb * c->per_batch;
        // largest h with QP * hp[h] <= r; heads without tiles are skipped by construction
        int lo = 0, hi = c->H - 1;
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if ((long long)c->QP * c->hp[mid] <= r) lo = mid;
            else hi = mid - 1;
        }
        const int nt = c->hp[lo + 1] - c->hp[lo];
        const long long r2 = r - (long long)c->QP * c->hp[lo];
        s.b = (int)bb;
        s.h = lo;
        s.nt = nt;
        s.qp = (int)(r2 / nt);
        s.j0 = (int)(r2 - (long long)s.qp * nt);
        const long long e = min(pos - s.j0 + nt, end);
        s.j1 = s.j0 + (int)(e - pos);
        pos = e;
        return true;
    }

    // CTAs above this one holding later parts of a unit whose first part ends this CTA's tail
    __device__ __noinline__ int partners(const Segment& s) const {
        const long long ue = bound((long long)blockIdx.x + 1) + (s.nt - s.j1);   // unit end
        int np = 0;
        while (np < kMaxPartners && (int)blockIdx.x + 1 + np < c->G_sk && bound((long long)blockIdx.x + 1 + np) < ue)
            ++np;
        return np;
    }
};

// Output store that the compiler does not treat as a memory clobber: the epilogue writes `out`
// (or this CTA's partial slot) and reads only another CTA's partial slot, which never overlap,
// so the partial loads may be scheduled ahead of these stores.
__device__ __forceinline__ void st_global_f2(float* ptr, float2 v) {
    asm volatile("st.global.v2.f32 [%0], {%1, %2};" ::"l"(ptr), "f"(v.x), "f"(v.y));
}

// Bounded wait (wall time) until `*flag` reaches `target` (acquire).
__device__ __forceinline__ bool wait_flag(const int* flag, int target, int* err, int code,
                                          uint64_t limit_ns = 1000000000ull) {
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t i = 0;; ++i) {
        int v;
        asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(flag) : "memory");
        if (v >= target) return true;
        __nanosleep(32);
        if ((i & 63) == 63) {
            if (*reinterpret_cast<volatile int*>(err) != 0) return false;
            if (globaltimer_ns() - t0 > limit_ns) {
                atomicCAS(err, 0, code);
                return false;
            }
        }
    }
}

// One float2 of the final output at element offset idx of the [B, H_out, S_q, D] layout: into
// every peer's buffer, or into `out`.
// With out_half the two values go out as one fp16 pair (round to nearest even).
__device__ __forceinline__ void st_global_h2(float* base, int64_t idx, float2 v) {
    const uint32_t h = half2_bits(__floats2half2_rn(v.x, v.y));
    asm volatile("st.global.b32 [%0], %1;" ::"l"(reinterpret_cast<__half*>(base) + idx), "r"(h));
}
template <bool PEERS>
__device__ __forceinline__ void out_store(const AttnParams& p, int64_t idx, float2 v) {
    if (!PEERS) {
        if (p.out_half)
            st_global_h2(p.out, idx, v);
        else
            st_global_f2(p.out + idx, v);
        return;
    }
    for (int r = 0; r < p.n_peers; ++r) {
        if (p.out_half)
            st_global_h2(p.peers[r], idx, v);
        else
            st_global_f2(p.peers[r] + idx, v);
    }
}

// Peer epilogue: a softmax warp stages 4 finished output rows -- contiguous in every rank's
// buffer -- in its shared-memory slot and sends them with one bulk copy per rank, so whole rows
// cross NVLink as large writes and the warp does not stall on remote stores.  The 16x256b TMEM
// share gives a warp 8 rows per pass (lane >> 2); the slot takes them in two halves, lanes
// 16 * sub .. 16 * sub + 15 (rows 4 * sub .. 4 * sub + 3), each pass reading O again.
// stage_acquire: the copies that read the slot last time have read it (the slot may be rewritten).
__device__ __forceinline__ void stage_acquire(int lane) {
    if (lane == 0) bulk_wait_read0();
    __syncwarp();
}
// this lane's two values of chunk c, part k of slot row (lane >> 2) & 3, when its row is in half `sub`
// (fp16 rows, half as long, when `half`)
template <int D>
__device__ __forceinline__ void stage_put(float* slot, bool half, int lane, int sub, int c, int k, float2 v) {
    if ((lane >> 4) != sub) return;
    const int e = ((lane >> 2) & 3) * D + c * 32 + 8 * k + 2 * (lane & 3);
    if (half)
        *reinterpret_cast<__half2*>(reinterpret_cast<__half*>(slot) + e) = __floats2half2_rn(v.x, v.y);
    else
        *reinterpret_cast<float2*>(slot + e) = v;
}
// slot rows [0, n) -> element idx of every rank's buffer
template <int D>
__device__ __noinline__ void stage_flush(const AttnParams& p, const float* slot, int lane, int64_t idx, int n) {
    fence_proxy_async_smem();
    __syncwarp();
    if (n <= 0) return;
    const int esz = p.out_half ? 2 : 4;
    for (int r = 0; r < p.n_peers; ++r) {
        uint8_t* g = reinterpret_cast<uint8_t*>(p.peers[r]) + idx * esz;
        if ((reinterpret_cast<uintptr_t>(g) & 15) == 0) {
            if (lane == 0) bulk_s2g(g, slot, (uint32_t)(n * D * esz));
        } else {
            const uint16_t* s16 = reinterpret_cast<const uint16_t*>(slot);
            for (int e = lane; e < n * D * esz / 2; e += 32) reinterpret_cast<uint16_t*>(g)[e] = s16[e];
        }
    }
    if (lane == 0) bulk_commit();
}

// Epilogue of a unit's first part when its later parts sit in np >= 2 other CTAs: rows rA and
// rB of this lane's 16x256b share, O = O_this * fa + sum_i O_i * 2^(m_i - m) / l_total, one
// partner at a time.  Kept out of line: the path is rare and its registers stay out of the
// softmax loop.  `o_empty` (may be null) gets the warp's arrival once O has been read out.
template <int D, bool PEERS>
__device__ __noinline__ void merge_parts(const AttnParams& p, uint32_t tO, int hf, int rA, int rB, float faA,
                                         float faB, float mA, float mB, float iA, float iB, int np, int slot, int rt,
                                         int lane, int nrows, int64_t obase, uint64_t* o_empty, float* oslot) {
    if constexpr (PEERS) {
        // rows rA (slot passes 0, 1) then rows rB (passes 2, 3), each staged and bulk-stored
#pragma unroll 1
        for (int pass = 0; pass < 4; ++pass) {
            const int half = pass >> 1, sub = pass & 1;
            const int r = half ? rB : rA;
            const float fr = half ? faB : faA, mr = half ? mB : mA, ir = half ? iB : iA;
            stage_acquire(lane);
#pragma unroll 1
            for (int c = 0; c < D / 32; ++c) {
                uint32_t o[16];
                tmem_ld16x256b_x4(tO + c * 32 + ((uint32_t)(hf * 16) << 16), o);
                tmem_wait_ld();
                if (o_empty != nullptr && hf == 1 && pass == 3 && c == D / 32 - 1) {
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(o_empty);
                }
                float2 v[4];
#pragma unroll
                for (int k = 0; k < 4; ++k)
                    v[k] = make_float2(__uint_as_float(o[4 * k + 2 * half]) * fr,
                                       __uint_as_float(o[4 * k + 2 * half + 1]) * fr);
                for (int i = 0; i < np; ++i) {
                    const size_t si2 = (size_t)(slot + i) * kUnitRows + rt;
                    const float f = ex2(__ldcg(p.part_ml + si2 + r).x - mr) * ir;
                    const float* srci = p.part_o + si2 * D;
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        const int col = c * 32 + 8 * k + 2 * (lane & 3);
                        const float2 x = __ldcg(reinterpret_cast<const float2*>(srci + (int64_t)r * D + col));
                        v[k] = make_float2(fmaf(x.x, f, v[k].x), fmaf(x.y, f, v[k].y));
                    }
                }
#pragma unroll
                for (int k = 0; k < 4; ++k) stage_put<D>(oslot, p.out_half, lane, sub, c, k, v[k]);
            }
            const int r0 = hf * 16 + half * 8 + sub * 4;
            stage_flush<D>(p, oslot, lane, obase + (int64_t)r0 * D, min(4, nrows - r0));
        }
        return;
    }
#pragma unroll 1
    for (int c = 0; c < D / 32; ++c) {
        uint32_t o[16];
        tmem_ld16x256b_x4(tO + c * 32 + ((uint32_t)(hf * 16) << 16), o);
        tmem_wait_ld();
        if (o_empty != nullptr && hf == 1 && c == D / 32 - 1) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(o_empty);
        }
        float2 va[4], vb[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            va[k] = make_float2(__uint_as_float(o[4 * k]) * faA, __uint_as_float(o[4 * k + 1]) * faA);
            vb[k] = make_float2(__uint_as_float(o[4 * k + 2]) * faB, __uint_as_float(o[4 * k + 3]) * faB);
        }
        for (int i = 0; i < np; ++i) {
            const size_t si2 = (size_t)(slot + i) * kUnitRows + rt;
            const float fA = ex2(__ldcg(p.part_ml + si2 + rA).x - mA) * iA;
            const float fB = ex2(__ldcg(p.part_ml + si2 + rB).x - mB) * iB;
            const float* srci = p.part_o + si2 * D;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int col = c * 32 + 8 * k + 2 * (lane & 3);
                const float2 xa = __ldcg(reinterpret_cast<const float2*>(srci + (int64_t)rA * D + col));
                const float2 xb = __ldcg(reinterpret_cast<const float2*>(srci + (int64_t)rB * D + col));
                va[k] = make_float2(fmaf(xa.x, fA, va[k].x), fmaf(xa.y, fA, va[k].y));
                vb[k] = make_float2(fmaf(xb.x, fB, vb[k].x), fmaf(xb.y, fB, vb[k].y));
            }
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int col = c * 32 + 8 * k + 2 * (lane & 3);
            if (rA < nrows) out_store<PEERS>(p, obase + (int64_t)rA * D + col, va[k]);
            if (rB < nrows) out_store<PEERS>(p, obase + (int64_t)rB * D + col, vb[k]);
        }
    }
}

// 2^x for a pair x <= 0 on the FMA pipe: x = n + f with n = rint(x) (the 1.5 * 2^23 rounding
// trick, exact for |x| < 2^22) and f in [-0.5, 0.5]; 2^f from a degree-3 polynomial whose
// coefficients were fitted here by a Remez exchange for minimax relative error on [-0.5, 0.5]
// (max 7.5e-5, below the fp16 rounding P gets next); n is added to the exponent field.  x is
// clamped at -126 so that the exponent stays in range (2^-126 is below every P that matters).
__device__ __forceinline__ float2 ex2_poly2(float2 x) {
    constexpr float kRound = 12582912.0f;   // 1.5 * 2^23
    x = make_float2(fmaxf(x.x, -126.0f), fmaxf(x.y, -126.0f));
    const float2 t = __fadd2_rn(x, make_float2(kRound, kRound));
    const float2 r = __fadd2_rn(t, make_float2(-kRound, -kRound));
    const float2 f = __ffma2_rn(r, make_float2(-1.0f, -1.0f), x);
    float2 q = __ffma2_rn(f, make_float2(0.0551716685f, 0.0551716685f), make_float2(0.2426111251f, 0.2426111251f));
    q = __ffma2_rn(q, f, make_float2(0.6932609677f, 0.6932609677f));
    q = __ffma2_rn(q, f, make_float2(0.9999280572f, 0.9999280572f));
    return make_float2(__int_as_float(__float_as_int(q.x) + (__float_as_int(t.x) << 23)),
                       __int_as_float(__float_as_int(q.y) + (__float_as_int(t.y) << 23)));
}

// Persistent, cooperatively launched (one CTA per SM, all resident): warps 0-7 softmax,
// warp 8 loader, warp 9 MMA issuer, as described at the top of this file, looping over the
// CTA's segments.  Barrier phases run on across segments (per step for the KV ring, S and P;
// per segment for Q and O), so the next unit's Q load and first S MMAs overlap the previous
// unit's epilogue.
// EMU: one column pair in four of every score row takes its exponentials from ex2_poly2 on the
// FMA pipe instead of the MUFU.
template <int D, bool PEERS, bool EMU>
__global__ void __launch_bounds__(kAttnThreads, 1)
    packed_attention_kernel(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ AttnParams p) {
    using L = AttnLayout<D, PEERS>;
    constexpr int NA = L::NA;
    constexpr uint32_t TB = L::kTile;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBar);
    uint64_t* q_full = bars;            // expect_tx arrive + TMA bytes, per segment
    uint64_t* q_empty = bars + 1;       // commit after the segment's last S MMAs
    uint64_t* k_full = bars + 2;        // [2] ring stages (K tile + lo tile of the selected channels)
    uint64_t* v_full = bars + 4;        // [2]
    uint64_t* k_empty = bars + 6;       // [2] commit
    uint64_t* v_empty = bars + 8;       // [2] commit
    uint64_t* s_full = bars + 10;       // [2] per query tile, commit
    uint64_t* p_full = bars + 12;       // [2] per query tile, 4 softmax warps
    uint64_t* o_full = bars + 14;       // [2] per query tile, commit after the segment's last P*V
    uint64_t* o_empty = bars + 16;      // [2] per query tile, 4 softmax warps (O read out)
    uint64_t* drain = bars + 18;        // commit, drain before TMEM release
    uint64_t* qc_full = bars + 19;      // loader warp: the segment's Q_c tiles are in shared memory
    SchedSmem* ss = reinterpret_cast<SchedSmem*>(smem + L::kSch);
    const int* hp = ss->hp;
    int* misc = reinterpret_cast<int*>(smem + L::kMisc);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kTmemSlot);

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        mbar_init(q_empty, 1);
        for (int s = 0; s < 2; ++s) {
            mbar_init(&k_full[s], 1);
            mbar_init(&v_full[s], 1);
            mbar_init(&k_empty[s], 1);
            mbar_init(&v_empty[s], 1);
            mbar_init(&s_full[s], 1);
            mbar_init(&p_full[s], 4);
            mbar_init(&o_full[s], 1);
            mbar_init(&o_empty[s], 4);
        }
        mbar_init(drain, 1);
        mbar_init(qc_full, 1);
        fence_mbarrier_init();
        Schedule::setup(ss, p);
    }
    if (warp == kMmaWarp) {
        tmem_alloc(tmem_slot, kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    Schedule sched;
    sched.init(ss);

    if (warp < kSoftmaxWarps) {
        // ------------------------------------------------------------------ softmax
        const int t = warp >> 2;                         // query tile of this warp group
        const int qw = warp & 3;                         // TMEM lane quarter: rows qw*32 + lane
        const uint32_t lane_off = (uint32_t)(qw * 32) << 16;
        const uint32_t tS = tmem + t * kBN + lane_off;
        const uint32_t tO = tmem + 2 * kBN + t * D + lane_off;
        const float sl2 = p.scale_log2;
        const int rt = t * kBM + qw * 32;                // first row of this warp in a unit
        Segment sg;
        long long g = 0;                                 // steps so far (KV tiles consumed)
        int si = 0;                                      // segments so far
        bool ok = true;
        while (ok && sched.next(sg)) {
            const int* cnt = p.counts + (int64_t)(sg.h / p.rep) * 5;
            const int n_stored = cnt[0] + cnt[1] + cnt[2] + cnt[3] + p.S_new;     // packed + dense rows
            const int n_ev = cnt[4];
            const bool first_part = sg.j0 == 0;
            // evicted rows (logit 0, no value) are counted once, by the unit's first part
            float m_ref = first_part && n_ev > 0 ? 0.0f : -INFINITY;
            float l = first_part ? (float)n_ev : 0.0f;
            for (int j = sg.j0; j < sg.j1; ++j, ++g) {
                if (!warp_wait(&s_full[t], (uint32_t)(g & 1), p.err, kErrSFull)) { ok = false; break; }
                tc_fence_after();
                uint32_t sc[kBN];
#pragma unroll
                for (int c = 0; c < kBN / 32; ++c)
                    tmem_ld32(tS + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&sc[c * 32]));
                tmem_wait_ld();
                // columns at or past n_valid hold no entry (past the head's last stored row)
                const int n_valid = n_stored - j * kBN;
                if (n_valid < kBN) {
#pragma unroll
                    for (int c = 0; c < kBN; ++c)
                        if (c >= n_valid) sc[c] = __float_as_uint(-INFINITY);
                }
                const float mt = row_max<kBN>(sc) * sl2;
                const bool need = mt > m_ref + kRescaleThreshold;
                const bool rescale = __any_sync(0xffffffffu, need);
                // rows that keep their reference max use factor 1 (TMEM access is warp-wide)
                const float fac = need ? ex2(m_ref - mt) : 1.0f;   // 0 when m_ref = -inf
                if (need) m_ref = mt;
                l *= fac;
                // P = 2^(s*scale - m_ref) in fp16, written over the first kBN/2 columns of S_t
                // (all of S_t is in registers by now)
                const float2 sl2x2 = make_float2(sl2, sl2), negm2 = make_float2(-m_ref, -m_ref);
                float2 acc0 = make_float2(0.f, 0.f), acc1 = make_float2(0.f, 0.f);
#pragma unroll
                for (int c = 0; c < kBN / 32; ++c) {
                    uint32_t pk[16];
#pragma unroll
                    for (int i = 0; i < 32; i += 2) {
                        const int col = c * 32 + i;
                        const float2 x = __ffma2_rn(
                            make_float2(__uint_as_float(sc[col]), __uint_as_float(sc[col + 1])), sl2x2, negm2);
                        const float2 e = (EMU && ((i >> 1) & 3) == 3) ? ex2_poly2(x) : make_float2(ex2(x.x), ex2(x.y));
                        if ((col >> 1) & 1)
                            acc1 = __fadd2_rn(acc1, e);
                        else
                            acc0 = __fadd2_rn(acc0, e);
                        pk[i / 2] = half2_bits(__floats2half2_rn(e.x, e.y));
                    }
                    tmem_st16(tS + c * 16, pk);
                }
                l += (acc0.x + acc0.y) + (acc1.x + acc1.y);
                if (rescale && j > sg.j0) {
                    // O_t holds this segment's tiles so far (s_full[t] was committed after the
                    // previous P_t V) and the next P_t V waits for p_full[t]: rescale it now
                    uint32_t o[32];
#pragma unroll
                    for (int c = 0; c < D / 32; ++c) {
                        tmem_ld32(tO + c * 32, o);
                        tmem_wait_ld();
#pragma unroll
                        for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * fac);
                        tmem_st32(tO + c * 32, o);
                    }
                }
                tmem_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&p_full[t]);
            }
            if (!ok) break;
            // ---------------------------------------------------------------- epilogue
            if (!warp_wait(&o_full[t], (uint32_t)(si & 1), p.err, kErrOFull)) { ok = false; break; }
            tc_fence_after();
            const bool split_tail = sg.j0 > 0;                   // a later part: publish, unnormalised
            const bool split_head = first_part && sg.j1 < sg.nt; // first part: merge the later parts
            // later parts live in CTAs blockIdx.x + 1 .. + np (each publishes into its own slot)
            const int np = split_head ? sched.partners(sg) : 0;
            const int slot = blockIdx.x + 1;
            float mB = -INFINITY, lB = 0.0f;
            for (int i = 0; i < np; ++i) {
                int got = 1;
                if (lane == 0) got = wait_flag(p.part_flag + slot + i, kSoftmaxWarps, p.err, kErrPartial) ? 1 : 0;
                got = __shfl_sync(0xffffffffu, got, 0);
                __syncwarp();
                if (!got) { ok = false; break; }
            }
            if (!ok) break;
            if (np == 1) {
                const float2 ml = __ldcg(p.part_ml + (size_t)slot * kUnitRows + rt + lane);
                mB = ml.x;
                lB = ml.y;
            }
            // per-row factors (thread = row): O = O_this * fa + O_other * fb
            float fa = 1.0f, fb = 0.0f;
            float mall = m_ref, inv_all = 0.0f;                  // np >= 2: common max and 1 / total
            if (!split_tail && np <= 1) {
                const float m = fmaxf(m_ref, mB);
                fa = m_ref == -INFINITY ? 0.0f : ex2(m_ref - m);
                fb = np == 1 ? ex2(mB - m) : 0.0f;
                const float lt = l * fa + lB * fb;
                const float inv = lt > 0.0f ? 1.0f / lt : 0.0f;
                fa *= inv;
                fb *= inv;
            } else if (!split_tail) {
                for (int i = 0; i < np; ++i)
                    mall = fmaxf(mall, __ldcg(p.part_ml + (size_t)(slot + i) * kUnitRows + rt + lane).x);
                float lt = m_ref == -INFINITY ? 0.0f : l * ex2(m_ref - mall);
                for (int i = 0; i < np; ++i) {
                    const float2 ml = __ldcg(p.part_ml + (size_t)(slot + i) * kUnitRows + rt + lane);
                    lt += ml.y * ex2(ml.x - mall);
                }
                inv_all = lt > 0.0f ? 1.0f / lt : 0.0f;
                fa = m_ref == -INFINITY ? 0.0f : ex2(m_ref - mall) * inv_all;
            }
            const int row0 = sg.qp * kUnitRows + rt;             // query row within the head
            const int64_t obase = (((int64_t)sg.b * p.H_out + p.head_off + sg.h) * p.S_q + row0) * D;
            float* dst = split_tail ? p.part_o + ((size_t)blockIdx.x * kUnitRows + rt) * D
                                    : p.out + (((int64_t)sg.b * p.H + sg.h) * p.S_q + row0) * D;
            const float* src = p.part_o + ((size_t)slot * kUnitRows + rt) * D;
            const int nrows = split_tail ? 32 : min(32, p.S_q - row0);
            // PEERS: this warp's staging slot (8 output rows)
            float* oslot = PEERS ? reinterpret_cast<float*>(smem + L::kOut) + warp * L::kOutRows * D : nullptr;
            // O is read in the 16x256b shape: four threads hold 32 contiguous bytes of a row, so
            // each store instruction writes whole sectors without a shared-memory transpose
            // (shared memory bandwidth stays with the tensor cores)
#pragma unroll 1
            for (int hf = 0; hf < 2; ++hf) {
                const int rA = hf * 16 + (lane >> 2), rB = rA + 8;
                const float faA = __shfl_sync(0xffffffffu, fa, rA), faB = __shfl_sync(0xffffffffu, fa, rB);
                const float fbA = __shfl_sync(0xffffffffu, fb, rA), fbB = __shfl_sync(0xffffffffu, fb, rB);
                if (np >= 2) {
                    // a unit spread over three or more CTAs (small grids of units)
                    const float mA = __shfl_sync(0xffffffffu, mall, rA), mBr = __shfl_sync(0xffffffffu, mall, rB);
                    const float iA = __shfl_sync(0xffffffffu, inv_all, rA), iB = __shfl_sync(0xffffffffu, inv_all, rB);
                    merge_parts<D, PEERS>(p, tO, hf, rA, rB, faA, faB, mA, mBr, iA, iB, np, slot, rt, lane, nrows, obase,
                                          &o_empty[t], oslot);
                    continue;
                }
                if (np == 1) {
                    if constexpr (PEERS) {
                        // rows rA, then rows rB, each in two slot halves: per row the partial
                        // values first (their loads overlap), then O chunk by chunk per pass
#pragma unroll 1
                        for (int half = 0; half < 2; ++half) {
                            const int r = half ? rB : rA;
                            const float fbr = half ? fbB : fbA, far = half ? faB : faA;
                            float2 px[D / 32][4];
#pragma unroll
                            for (int c = 0; c < D / 32; ++c)
#pragma unroll
                                for (int k = 0; k < 4; ++k)
                                    px[c][k] = __ldcg(reinterpret_cast<const float2*>(
                                        src + (int64_t)r * D + c * 32 + 8 * k + 2 * (lane & 3)));
#pragma unroll 1
                            for (int sub = 0; sub < 2; ++sub) {
                                stage_acquire(lane);
#pragma unroll
                                for (int c = 0; c < D / 32; ++c) {
                                    uint32_t o[16];
                                    tmem_ld16x256b_x4(tO + c * 32 + ((uint32_t)(hf * 16) << 16), o);
                                    tmem_wait_ld();
                                    if (hf == 1 && half == 1 && sub == 1 && c == D / 32 - 1) {
                                        tc_fence_before();
                                        __syncwarp();
                                        if (lane == 0) mbar_arrive(&o_empty[t]);
                                    }
#pragma unroll
                                    for (int k = 0; k < 4; ++k)
                                        stage_put<D>(oslot, p.out_half, lane, sub, c, k,
                                                     make_float2(fmaf(px[c][k].x, fbr, __uint_as_float(o[4 * k + 2 * half]) * far),
                                                                 fmaf(px[c][k].y, fbr, __uint_as_float(o[4 * k + 2 * half + 1]) * far)));
                                }
                                const int r0 = hf * 16 + half * 8 + sub * 4;
                                stage_flush<D>(p, oslot, lane, obase + (int64_t)r0 * D, min(4, nrows - r0));
                            }
                        }
                        continue;
                    }
                    // a unit cut between two CTAs, merged here (once per CTA at most): all of this
                    // half's partial values first, so their loads overlap, then O chunk by chunk
                    float2 pa[D / 32][4], pb[D / 32][4];
#pragma unroll
                    for (int c = 0; c < D / 32; ++c)
#pragma unroll
                        for (int k = 0; k < 4; ++k) {
                            const int col = c * 32 + 8 * k + 2 * (lane & 3);
                            pa[c][k] = __ldcg(reinterpret_cast<const float2*>(src + (int64_t)rA * D + col));
                            pb[c][k] = __ldcg(reinterpret_cast<const float2*>(src + (int64_t)rB * D + col));
                        }
#pragma unroll
                    for (int c = 0; c < D / 32; ++c) {
                        uint32_t o[16];
                        tmem_ld16x256b_x4(tO + c * 32 + ((uint32_t)(hf * 16) << 16), o);
                        tmem_wait_ld();
                        if (hf == 1 && c == D / 32 - 1) {
                            tc_fence_before();
                            __syncwarp();
                            if (lane == 0) mbar_arrive(&o_empty[t]);
                        }
#pragma unroll
                        for (int k = 0; k < 4; ++k) {
                            const int col = c * 32 + 8 * k + 2 * (lane & 3);
                            const float2 va = make_float2(fmaf(pa[c][k].x, fbA, __uint_as_float(o[4 * k]) * faA),
                                                          fmaf(pa[c][k].y, fbA, __uint_as_float(o[4 * k + 1]) * faA));
                            const float2 vb = make_float2(fmaf(pb[c][k].x, fbB, __uint_as_float(o[4 * k + 2]) * faB),
                                                          fmaf(pb[c][k].y, fbB, __uint_as_float(o[4 * k + 3]) * faB));
                            if (rA < nrows) out_store<PEERS>(p, obase + (int64_t)rA * D + col, va);
                            if (rB < nrows) out_store<PEERS>(p, obase + (int64_t)rB * D + col, vb);
                        }
                    }
                    continue;
                }
                if constexpr (PEERS) {
                    if (!split_tail) {
                        // rows rA, then rows rB, each in two slot halves; O read chunk by chunk
                        // per pass so that few registers stay live beside the bulk-store issue
#pragma unroll 1
                        for (int pass = 0; pass < 4; ++pass) {
                            const int half = pass >> 1, sub = pass & 1;
                            const float fr = half ? faB : faA;
                            stage_acquire(lane);
#pragma unroll
                            for (int c = 0; c < D / 32; ++c) {
                                uint32_t o[16];
                                tmem_ld16x256b_x4(tO + c * 32 + ((uint32_t)(hf * 16) << 16), o);
                                tmem_wait_ld();
                                if (hf == 1 && pass == 3 && c == D / 32 - 1) {
                                    tc_fence_before();
                                    __syncwarp();
                                    if (lane == 0) mbar_arrive(&o_empty[t]);
                                }
#pragma unroll
                                for (int k = 0; k < 4; ++k)
                                    stage_put<D>(oslot, p.out_half, lane, sub, c, k,
                                                 make_float2(__uint_as_float(o[4 * k + 2 * half]) * fr,
                                                             __uint_as_float(o[4 * k + 2 * half + 1]) * fr));
                            }
                            const int r0 = hf * 16 + half * 8 + sub * 4;
                            stage_flush<D>(p, oslot, lane, obase + (int64_t)r0 * D, min(4, nrows - r0));
                        }
                        continue;
                    }
                }
                // all of this half's TMEM columns first (one wait), then the stores
                uint32_t o[D / 32][16];
#pragma unroll
                for (int c = 0; c < D / 32; ++c)
                    tmem_ld16x256b_x4(tO + c * 32 + ((uint32_t)(hf * 16) << 16), o[c]);
                tmem_wait_ld();
                if (hf == 1) {
                    // O_t has been read out: the next segment's first P_t V may overwrite it
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&o_empty[t]);
                }
#pragma unroll
                for (int c = 0; c < D / 32; ++c) {
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        const int col = c * 32 + 8 * k + 2 * (lane & 3);
                        const float2 va = make_float2(__uint_as_float(o[c][4 * k]) * faA, __uint_as_float(o[c][4 * k + 1]) * faA);
                        const float2 vb = make_float2(__uint_as_float(o[c][4 * k + 2]) * faB, __uint_as_float(o[c][4 * k + 3]) * faB);
                        if (split_tail) {
                            // published to another CTA behind a fence: ordinary stores
                            *reinterpret_cast<float2*>(dst + (int64_t)rA * D + col) = va;
                            *reinterpret_cast<float2*>(dst + (int64_t)rB * D + col) = vb;
                        } else {
                            if (rA < nrows) out_store<PEERS>(p, obase + (int64_t)rA * D + col, va);
                            if (rB < nrows) out_store<PEERS>(p, obase + (int64_t)rB * D + col, vb);
                        }
                    }
                }
            }
            if (split_tail) {
                p.part_ml[(size_t)blockIdx.x * kUnitRows + rt + lane] = make_float2(m_ref, l);
                __threadfence();
                __syncwarp();
                if (lane == 0) atomicAdd(p.part_flag + blockIdx.x, 1);
            }
            ++si;
        }
        // units of heads without a stored entry are never scheduled: their output is zero
        const long long U = (long long)p.B * p.H * p.QP;
        for (long long u = blockIdx.x; u < U; u += gridDim.x) {
            const int qp = (int)(u % p.QP);
            const int hh = (int)((u / p.QP) % p.H);
            const int bb = (int)(u / ((long long)p.QP * p.H));
            if (hp[hh + 1] != hp[hh]) continue;
            const int row0 = qp * kUnitRows + rt;
            const int64_t ob = (((int64_t)bb * p.H_out + p.head_off + hh) * p.S_q + row0) * D;
            for (int r = 0; r < min(32, p.S_q - row0); ++r)
                for (int d = 2 * lane; d < D; d += 64) out_store<PEERS>(p, ob + (int64_t)r * D + d, make_float2(0.0f, 0.0f));
        }
        if constexpr (PEERS) {
            // the staged rows' bulk stores have completed before the CTA (and its shared memory) ends
            if (lane == 0) bulk_wait0();
            __syncwarp();
        }
    } else if (warp == kLoadWarp) {
        // ------------------------------------------------------------------ loader
        // Lane 0 issues every copy; with the lo correction the whole warp then gathers the
        // segment's Q_c tiles (the queries' selected channels) from the Q tiles once they land.
        Segment sg;
        long long g = 0;
        int si = 0, nq = 0;
        int nk[2] = {0, 0}, nv[2] = {0, 0};          // copies issued per stage (lane 0)
        bool ok = true;
        // lane 0 waits, the warp agrees on the outcome
        auto lane0_wait = [&](uint64_t* bar, uint32_t parity, int code) -> bool {
            int r = 1;
            if (lane == 0) r = mbar_wait_spin(bar, parity, p.err, code) ? 1 : 0;
            return __shfl_sync(0xffffffffu, r, 0) != 0;
        };
        while (ok && sched.next(sg)) {
            if (si > 0 && !lane0_wait(q_empty, (uint32_t)((si - 1) & 1), kErrQEmpty)) break;
            const int qrow = (sg.b * p.H + sg.h) * p.S_q + sg.qp * kUnitRows;
            if (lane == 0) {
                mbar_arrive_expect_tx(q_full, 2 * TB);
#pragma unroll
                for (int t = 0; t < 2; ++t)
#pragma unroll
                    for (int a = 0; a < NA; ++a)
                        tma_load_2d(smem + L::kQ + t * TB + a * kBM * 128, &qmap, a * 64, qrow + t * kBM, q_full);
            }
            ++nq;
            const uint8_t* gkv = p.stage + staged_offset(p, sg.b, sg.h / p.rep, 0, D);
            HeadRows hr;
            hr.load(p, sg.h);
            const int selc = p.klo && lane < kLoCh ? __ldg(p.sel + (int64_t)(sg.h / p.rep) * kLoCh + lane) : 0;
            for (int j = sg.j0; j < sg.j1; ++j, ++g) {
                const int s = (int)(g & 1);
                const uint8_t* set = gkv + (int64_t)j * staged_set_bytes(D);
                if (g >= 2 && !lane0_wait(&k_empty[s], (uint32_t)(((g >> 1) - 1) & 1), kErrKEmpty)) {
                    ok = false;
                    break;
                }
                if (lane == 0) {
                    // K and, unless the tile is exact in fp16, the lo tile of the selected channels
                    const bool lo = !hr.exact(j);
                    mbar_arrive_expect_tx(&k_full[s], lo ? TB + kLoTile : TB);
                    bulk_g2s(smem + L::kK + s * TB, set, TB, &k_full[s]);
                    if (lo) bulk_g2s(smem + L::kKc + s * kLoTile, set + 2 * TB, kLoTile, &k_full[s]);
                    ++nk[s];
                }
                if (g >= 2 && !lane0_wait(&v_empty[s], (uint32_t)(((g >> 1) - 1) & 1), kErrVEmpty)) {
                    ok = false;
                    break;
                }
                if (lane == 0) {
                    mbar_arrive_expect_tx(&v_full[s], TB);
                    bulk_g2s(smem + L::kV + s * TB, set + TB, TB, &v_full[s]);
                    ++nv[s];
                }
                if (j == sg.j0 && p.klo) {
                    // Q_c: the selected channels of both query tiles, 32-byte-swizzled rows.  The
                    // previous segment's S MMAs (the last readers of Q_c) completed before q_empty.
                    if (!warp_wait(q_full, (uint32_t)(si & 1), p.err, kErrQFull)) {
                        ok = false;
                        break;
                    }
                    int sc[kLoCh];
#pragma unroll
                    for (int i = 0; i < kLoCh; ++i) sc[i] = __shfl_sync(0xffffffffu, selc, i) & (D - 1);  // in the tile
#pragma unroll 1
                    for (int t = 0; t < 2; ++t) {
                        const uint8_t* qt = smem + L::kQ + t * TB;
                        uint8_t* qc = smem + L::kQc + t * kLoTile;
#pragma unroll 1
                        for (int r = lane; r < kBM; r += 32) {
                            uint32_t w[kLoCh / 2];
#pragma unroll
                            for (int i = 0; i < kLoCh; i += 2) {
                                const int c0 = sc[i], c1 = sc[i + 1];
                                const uint32_t lo16 = *reinterpret_cast<const uint16_t*>(
                                    qt + (c0 >> 6) * (kBM * 128) + sw128_offset(r, (c0 & 63) >> 3) + (c0 & 7) * 2);
                                const uint32_t hi16 = *reinterpret_cast<const uint16_t*>(
                                    qt + (c1 >> 6) * (kBM * 128) + sw128_offset(r, (c1 & 63) >> 3) + (c1 & 7) * 2);
                                w[i / 2] = lo16 | (hi16 << 16);
                            }
                            *reinterpret_cast<uint4*>(qc + sw32_offset(r, 0)) = make_uint4(w[0], w[1], w[2], w[3]);
                            *reinterpret_cast<uint4*>(qc + sw32_offset(r, 1)) = make_uint4(w[4], w[5], w[6], w[7]);
                        }
                    }
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(qc_full);
                }
            }
            ++si;
        }
        if (lane == 0) {
            // every copy issued lands before the CTA can exit (a no-op when the MMA consumed them)
            if (nq) mbar_wait_spin(q_full, (uint32_t)((nq - 1) & 1), p.err, kErrCopy);
            for (int s = 0; s < 2; ++s) {
                if (nk[s]) mbar_wait_spin(&k_full[s], (uint32_t)((nk[s] - 1) & 1), p.err, kErrCopy);
                if (nv[s]) mbar_wait_spin(&v_full[s], (uint32_t)((nv[s] - 1) & 1), p.err, kErrCopy);
            }
        }
        __syncwarp();
    } else {
        // ----------------------------------------------------------------- MMA issue
        if (lane == 0) {
            const uint32_t idesc_s = idesc_f16_f32(kBM, kBN, false, false);
            const uint32_t idesc_o = idesc_f16_f32(kBM, D, false, true);
            // Shared-memory descriptors of the operands, built once: the descriptor of address
            // a + off is the descriptor of a plus off / 16 (shared addresses stay below 2^18, so
            // the 14-bit address field never carries), so an MMA costs one add per operand.
            const uint64_t qd0 = smem_desc_sw128(smem_u32(smem + L::kQ), 16, 1024);
            const uint64_t kd0 = smem_desc_sw128(smem_u32(smem + L::kK), 16, 1024);
            const uint64_t vd0 = smem_desc_sw128(smem_u32(smem + L::kV), kBN * 128, 1024);
            const uint64_t qcd0 = smem_desc_sw32(smem_u32(smem + L::kQc), 16, 256);
            const uint64_t kcd0 = smem_desc_sw32(smem_u32(smem + L::kKc), 16, 256);
            // K stage of step g and the parity of its full barrier
            auto kstage = [&](long long g) { return (int)(g & 1); };
            auto kparity = [&](long long g) { return (uint32_t)((g >> 1) & 1); };
            // S_t = Q_t K^T (fp16), then += Q_c,t K_lo^T over the selected channels (one K = 16 step)
            // unless the tile is exact in fp16
            auto issue_s = [&](int t, long long g, bool lo) {
                const uint64_t qd = qd0 + (uint64_t)((t * TB) >> 4);
                const uint64_t kd = kd0 + (uint64_t)((kstage(g) * TB) >> 4);
                const uint32_t d = tmem + t * kBN;
#pragma unroll
                for (int k = 0; k < D / 16; ++k) {
                    const uint64_t off = (uint64_t)((((k >> 2) * (kBN * 128)) + (k & 3) * 32) >> 4);
                    if (k == 0)
                        umma_f16(d, qd + off, kd + off, idesc_s, 0u);
                    else
                        umma_f16_acc(d, qd + off, kd + off, idesc_s);
                }
                if (lo)
                    umma_f16_acc(d, qcd0 + (uint64_t)((t * kLoTile) >> 4), kcd0 + (uint64_t)((kstage(g) * kLoTile) >> 4),
                                 idesc_s);
            };
            auto issue_pv = [&](int t, long long g, bool acc) {
                const uint64_t vd = vd0 + (uint64_t)(((int)(g & 1) * TB) >> 4);
                const uint32_t d = tmem + 2 * kBN + t * D, a = tmem + t * kBN;
#pragma unroll
                for (int k = 0; k < kBN / 16; ++k) {
                    if (k == 0)
                        umma_f16_ts(d, a, vd, idesc_o, acc ? 1u : 0u);
                    else
                        umma_f16_ts_acc(d, a + k * 8, vd + (uint64_t)((k * 16 * 128) >> 4), idesc_o);
                }
            };
            Segment sg;
            long long g = 0;
            int si = 0;
            bool ok = true, issued = false;
            while (ok && sched.next(sg)) {
                const int len = sg.j1 - sg.j0;
                HeadRows hr;
                hr.load(p, sg.h);
                if (!mbar_wait_spin(q_full, (uint32_t)(si & 1), p.err, kErrQFull) ||
                    (p.klo && !mbar_wait_spin(qc_full, (uint32_t)(si & 1), p.err, kErrQFull)) ||
                    !mbar_wait_spin(&k_full[kstage(g)], kparity(g), p.err, kErrKFull)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                // S of the segment's first step; P_t of the previous segment's last step has
                // been read by its P_t V, issued before (the tensor pipe runs in issue order)
                const bool lo0 = !hr.exact(sg.j0);
                issue_s(0, g, lo0);
                umma_commit(&s_full[0]);
                issue_s(1, g, lo0);
                umma_commit(&s_full[1]);
                umma_commit(&k_empty[kstage(g)]);
                if (len == 1) umma_commit(q_empty);
                issued = true;
                for (int j = 0; j < len; ++j, ++g) {
                    const int s = (int)(g & 1);
                    const bool more = j + 1 < len;
                    const bool lo1 = more && !hr.exact(sg.j0 + j + 1);
                    // every operand of P_0 V and of the next S_0 before either is issued: a wait
                    // between the two batches would let the tensor pipe run dry (a barrier wait
                    // costs the issuing thread as long as the MMAs it could have queued)
                    if (!mbar_wait_spin(&v_full[s], (uint32_t)((g >> 1) & 1), p.err, kErrVFull) ||
                        (more && !mbar_wait_spin(&k_full[kstage(g + 1)], kparity(g + 1), p.err, kErrKFull)) ||
                        (j == 0 && si > 0 && !mbar_wait_spin(&o_empty[0], (uint32_t)((si - 1) & 1), p.err, kErrOEmpty)) ||
                        !mbar_wait_spin(&p_full[0], (uint32_t)(g & 1), p.err, kErrPFull)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    issue_pv(0, g, j > 0);
                    if (!more) umma_commit(&o_full[0]);
                    if (more) {
                        // issued after P_0 V: the tensor pipe has read P_0 before S_0 is rewritten
                        issue_s(0, g + 1, lo1);
                        umma_commit(&s_full[0]);
                    }
                    if (!mbar_wait_spin(&p_full[1], (uint32_t)(g & 1), p.err, kErrPFull) ||
                        (j == 0 && si > 0 && !mbar_wait_spin(&o_empty[1], (uint32_t)((si - 1) & 1), p.err, kErrOEmpty))) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    issue_pv(1, g, j > 0);
                    umma_commit(&v_empty[s]);
                    if (!more) umma_commit(&o_full[1]);
                    if (more) {
                        issue_s(1, g + 1, lo1);
                        umma_commit(&s_full[1]);
                        umma_commit(&k_empty[kstage(g + 1)]);
                        if (j + 2 == len) umma_commit(q_empty);
                    }
                }
                ++si;
            }
            if (issued) {
                // drain: every UMMA issued above completes before TMEM is released
                umma_commit(drain);
                mbar_wait_spin(drain, 0, p.err, kErrDrain);
            }
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



#include "attention_1t.cuh"
#include "attention_pair.cuh"

// ---------------------------------------------------------------------------------------
// per-head row index
// ---------------------------------------------------------------------------------------
constexpr int kHiThreads = 1024;

// Grid (chunks, H): block (c, h) first counts every token of head h per code -- the totals give
// where each code's run of rows starts, the counts of the tokens before its chunk its offset
// inside each run -- and then writes the rows of the stored entries of its chunk of tokens
// (C tokens, a multiple of the block size) in token order: ballots per warp, an exclusive scan
// of the warps' counts by warp 0, one pass of the block per 1024 tokens.  Splitting a head over
// several blocks keeps the kernel short when there are few heads (a head-sharded rank).
__global__ void __launch_bounds__(kHiThreads) head_index_kernel(const int32_t* __restrict__ slot, int S, int H, int C,
                                                                int32_t* __restrict__ rows, int32_t* __restrict__ counts) {
    constexpr int NW = kHiThreads / 32;
    const int h = blockIdx.y;
    const int t_begin = blockIdx.x * C, t_end = min(S, t_begin + C);
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    __shared__ int s_red[9][NW];     // per warp: totals of codes 0-4, then codes 0-3 before the chunk
    __shared__ int s_run[4];
    __shared__ int s_cnt[4][NW];
    __shared__ int s_pre[4][NW];
    __shared__ int s_tot[4];
    int c[9] = {0, 0, 0, 0, 0, 0, 0, 0, 0};
    for (int t = threadIdx.x; t < S; t += kHiThreads) {
        const int32_t sl = slot[(int64_t)t * H + h];
        const int code = sl < 0 ? 4 : slot_code(sl);
        const bool before = t < t_begin;
#pragma unroll
        for (int k = 0; k < 5; ++k) c[k] += code == k;
#pragma unroll
        for (int k = 0; k < 4; ++k) c[5 + k] += (code == k) & before;
    }
#pragma unroll
    for (int k = 0; k < 9; ++k) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) c[k] += __shfl_xor_sync(0xffffffffu, c[k], o);
    }
    if (lane == 0) {
#pragma unroll
        for (int k = 0; k < 9; ++k) s_red[k][w] = c[k];
    }
    __syncthreads();
    if (w == 0) {
        // lane k < 9: the block's sum of row k
        int v = 0;
        if (lane < 9)
            for (int q = 0; q < NW; ++q) v += s_red[lane][q];
        const int t0 = __shfl_sync(0xffffffffu, v, 0), t1 = __shfl_sync(0xffffffffu, v, 1);
        const int t2 = __shfl_sync(0xffffffffu, v, 2);
        const int b = __shfl_sync(0xffffffffu, v, (lane & 3) + 5);     // code (lane & 3) before the chunk
        if (lane < 4) {
            // code k's run starts after the rows of codes 0 .. k-1
            const int start = lane == 0 ? 0 : (lane == 1 ? t0 : (lane == 2 ? t0 + t1 : t0 + t1 + t2));
            s_run[lane] = start + b;
        }
        if (blockIdx.x == 0 && lane < 5) counts[(int64_t)h * 5 + lane] = v;
    }
    __syncthreads();
    int r0 = s_run[0], r1 = s_run[1], r2 = s_run[2], r3 = s_run[3];
    for (int t0 = t_begin; t0 < t_end; t0 += kHiThreads) {
        const int t = t0 + threadIdx.x;
        const int32_t sl = t < t_end ? slot[(int64_t)t * H + h] : -1;
        const int code = sl < 0 ? 4 : slot_code(sl);
        const unsigned m0 = __ballot_sync(0xffffffffu, code == 0);
        const unsigned m1 = __ballot_sync(0xffffffffu, code == 1);
        const unsigned m2 = __ballot_sync(0xffffffffu, code == 2);
        const unsigned m3 = __ballot_sync(0xffffffffu, code == 3);
        if (lane == 0) {
            s_cnt[0][w] = __popc(m0);
            s_cnt[1][w] = __popc(m1);
            s_cnt[2][w] = __popc(m2);
            s_cnt[3][w] = __popc(m3);
        }
        __syncthreads();
        if (w < 4) {
            // warp k: exclusive scan of code k's counts over the warps
            const int v = lane < NW ? s_cnt[w][lane] : 0;
            int incl = v;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int u = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += u;
            }
            if (lane < NW) s_pre[w][lane] = incl - v;
            if (lane == 31) s_tot[w] = incl;
        }
        __syncthreads();
        if (code < 4) {
            const unsigned m = code == 0 ? m0 : (code == 1 ? m1 : (code == 2 ? m2 : m3));
            const int run = code == 0 ? r0 : (code == 1 ? r1 : (code == 2 ? r2 : r3));
            rows[(int64_t)h * S + run + s_pre[code][w] + __popc(m & ((1u << lane) - 1u))] = sl;
        }
        r0 += s_tot[0];
        r1 += s_tot[1];
        r2 += s_tot[2];
        r3 += s_tot[3];
        __syncthreads();
    }
}

}  // namespace skv

using namespace skv;

extern "C" {

int skv_head_index(const int32_t* slot, int S, int H, int32_t* rows, int32_t* counts, void* stream) {
    if (!slot || !rows || !counts) return fail(SKV_ERR_INVALID_ARGUMENT, "head_index: null pointer");
    if (S <= 0 || H <= 0) return fail(SKV_ERR_INVALID_ARGUMENT, "head_index: bad shape");
    // chunks of whole 1024-token passes, enough of them for ~two blocks per SM in all
    const int passes = (S + kHiThreads - 1) / kHiThreads;
    const int want = std::max(1, std::min(passes, (2 * sm_count() + H - 1) / H));
    const int C = (passes + want - 1) / want * kHiThreads;
    const int nchunks = (S + C - 1) / C;
    if (H > 65535) return fail(SKV_ERR_TOO_LARGE, "head_index: more than 65535 heads");
    head_index_kernel<<<dim3(nchunks, H), kHiThreads, 0, as_stream(stream)>>>(slot, S, H, C, rows, counts);
    return check_launch("head_index");
}

// Bytes of the per-KV-head channel maxima (uint32 [H, D]) and selected channels (int32 [H, kLoCh]),
// each rounded up to 256 bytes.
static size_t chan_bytes(int H, int D) {
    return (((size_t)H * D * 4 + 255) & ~size_t(255)) + (((size_t)H * kLoCh * 4 + 255) & ~size_t(255));
}

size_t skv_packed_attention_scratch_bytes(int B, int H, int S_kv, int D) {
    if (B <= 0 || H <= 0 || S_kv <= 0 || (D != 64 && D != 128)) return 0;
    const size_t ntmax = (size_t)(S_kv + kBN - 1) / kBN;
    const size_t slots = (size_t)sm_count();
    return (size_t)B * H * ntmax * staged_set_bytes(D)                // staged K, V, K lo tiles
           + chan_bytes(H, D)                                          // channel maxima, selection
           + slots * kUnitRows * D * sizeof(float)                    // partial O
           + slots * kUnitRows * sizeof(float2)                       // partial (max, sum)
           + ((slots * sizeof(int) + 255) & ~size_t(255));            // partial flags
}

}  // extern "C"

namespace {

int attn_params(const void* q, int B, int H, int S_q, int D, const skv_bucket* buckets, int H_kv, int S_kv,
                int int4_group, const int32_t* rows, const int32_t* counts, const float* k_new, const float* v_new,
                int S_new, float scale, void* scratch, size_t scratch_bytes, float* out, int32_t* error_flag,
                AttnParams& prm, const char* what, int max_ctas = 0, float* const* peers = nullptr,
                int n_peers = 0, int head_off = 0, int H_out = 0, int flags = 0) {
    if (!rows || !counts || !scratch) return fail(SKV_ERR_INVALID_ARGUMENT, "%s: null pointer", what);
    if (flags & ~(SKV_ATTN_FAST_K | SKV_ATTN_ONE_TILE | SKV_ATTN_FMA_EXP | SKV_ATTN_PAIR | SKV_ATTN_OUT_F16))
        return fail(SKV_ERR_INVALID_ARGUMENT, "%s: unknown flags 0x%x", what, flags);
    if ((flags & SKV_ATTN_PAIR) && (flags & (SKV_ATTN_ONE_TILE | SKV_ATTN_FMA_EXP)))
        return fail(SKV_ERR_INVALID_ARGUMENT, "%s: the CTA-pair pipeline takes no other pipeline flag", what);
    if (B <= 0 || H <= 0 || S_q <= 0 || S_kv <= 0 || H_kv <= 0 || S_new < 0)
        return fail(SKV_ERR_INVALID_ARGUMENT, "%s: bad shape", what);
    if (H % H_kv) return fail(SKV_ERR_SHAPE, "%s: %d query heads do not group over %d KV heads", what, H, H_kv);
    if (S_new > 0 && (!k_new || !v_new)) return fail(SKV_ERR_INVALID_ARGUMENT, "%s: null new K/V", what);
    if (S_new > 0 && ((reinterpret_cast<uintptr_t>(k_new) | reinterpret_cast<uintptr_t>(v_new)) & 15))
        return fail(SKV_ERR_UNSUPPORTED, "%s: new K/V not 16-byte aligned", what);
    if (D != 64 && D != 128) return fail(SKV_ERR_UNSUPPORTED, "%s: head_dim %d (64 or 128 supported)", what, D);
    const int G = int4_group > 0 && D % int4_group == 0 ? int4_group : D;
    if (G % 8) return fail(SKV_ERR_UNSUPPORTED, "%s: int4 group %d must be a multiple of 8", what, G);
    if (buckets) {
        for (int p = 0; p < kNumBuckets; ++p) {
            if (buckets[p].count == 0) continue;
            const uintptr_t a = reinterpret_cast<uintptr_t>(buckets[p].k) | reinterpret_cast<uintptr_t>(buckets[p].v);
            if (a & 15) return fail(SKV_ERR_UNSUPPORTED, "%s: bucket %d not 16-byte aligned", what, p);
        }
    }
    if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(out) | reinterpret_cast<uintptr_t>(scratch)) & 15)
        return fail(SKV_ERR_UNSUPPORTED, "%s: q/out/scratch not 16-byte aligned", what);
    const size_t need = skv_packed_attention_scratch_bytes(B, H_kv, S_kv + S_new, D);
    if (scratch_bytes < need)
        return fail(SKV_ERR_SCRATCH, "%s: scratch of %zu bytes, %zu needed", what, scratch_bytes, need);
    if ((long long)B * H * S_q >= (1ll << 31) || H > kMaxHeads ||
        (long long)H * ((S_kv + S_new + kBN - 1) / kBN) >= (1ll << 31))
        return fail(SKV_ERR_TOO_LARGE, "%s: B*H*S_q and H*ceil((S_kv+S_new)/128) must stay below 2^31, H <= %d",
                    what, kMaxHeads);
    memset(&prm, 0, sizeof(prm));
    prm.q = reinterpret_cast<const __half*>(q);
    prm.out = out;
    if (buckets)
        for (int p = 0; p < kNumBuckets; ++p) prm.bk.b[p] = buckets[p];
    prm.rows = rows;
    prm.counts = counts;
    prm.k_new = S_new > 0 ? k_new : nullptr;
    prm.v_new = S_new > 0 ? v_new : nullptr;
    prm.H_kv = H_kv;
    prm.rep = H / H_kv;
    prm.peers = n_peers > 0 ? peers : nullptr;
    prm.n_peers = n_peers > 0 ? n_peers : 0;
    prm.head_off = n_peers > 0 ? head_off : 0;
    prm.H_out = n_peers > 0 ? H_out : H;
    prm.S_new = S_new;
    prm.stage = reinterpret_cast<uint8_t*>(scratch);
    prm.ntmax = (S_kv + S_new + kBN - 1) / kBN;
    prm.slots = max_ctas > 0 && max_ctas < sm_count() ? max_ctas : sm_count();
    uint8_t* part = prm.stage + (size_t)B * H_kv * prm.ntmax * staged_set_bytes(D);
    prm.chmax = reinterpret_cast<unsigned*>(part);
    prm.sel = reinterpret_cast<int*>(part + (((size_t)H_kv * D * 4 + 255) & ~size_t(255)));
    part += chan_bytes(H_kv, D);
    prm.part_o = reinterpret_cast<float*>(part);
    part += (size_t)prm.slots * kUnitRows * D * sizeof(float);
    prm.part_ml = reinterpret_cast<float2*>(part);
    part += (size_t)prm.slots * kUnitRows * sizeof(float2);
    prm.part_flag = reinterpret_cast<int*>(part);
    prm.B = B;
    prm.H = H;
    prm.S_q = S_q;
    prm.S_kv = S_kv;
    prm.G = G;
    prm.one_tile = (flags & SKV_ATTN_ONE_TILE) ? 1 : 0;
    prm.pair = (flags & SKV_ATTN_PAIR) ? 1 : 0;
    prm.out_half = (flags & SKV_ATTN_OUT_F16) ? 1 : 0;
    prm.emu = (flags & SKV_ATTN_FMA_EXP) ? 1 : 0;
    prm.QP = prm.one_tile ? (S_q + k1TUnitRows - 1) / k1TUnitRows : (S_q + kUnitRows - 1) / kUnitRows;
    prm.scale_log2 = scale * 1.4426950408889634f;
    prm.err = error_flag;
    prm.klo = (flags & SKV_ATTN_FAST_K) ? 0 : 1;
    return SKV_OK;
}

}  // namespace

extern "C" {

int skv_stage_kv_tiles_gqa(const skv_bucket* buckets, int B, int H_kv, int S_kv, int D, int int4_group,
                           const int32_t* rows, const int32_t* counts, const float* k_new, const float* v_new,
                           int S_new, void* scratch, size_t scratch_bytes, int flags, void* stream) {
    if (!buckets) return fail(SKV_ERR_INVALID_ARGUMENT, "stage_kv_tiles: null pointer");
    AttnParams prm;
    const int st = attn_params(nullptr, B, H_kv, 1, D, buckets, H_kv, S_kv, int4_group, rows, counts, k_new, v_new,
                               S_new, 1.0f, scratch, scratch_bytes, nullptr, nullptr, prm, "stage_kv_tiles", 0,
                               nullptr, 0, 0, 0, flags);
    if (st != SKV_OK) return st;
    const dim3 grid((unsigned)prm.ntmax, (unsigned)H_kv, (unsigned)B);
    cudaStream_t s = as_stream(stream);
    if (prm.klo) {
        // the kLoCh channels of largest max |K| per KV head, whose lo parts are staged
        if (cudaMemsetAsync(prm.chmax, 0, (size_t)H_kv * D * 4, s) != cudaSuccess)
            return fail(SKV_ERR_CUDA, "stage_kv_tiles: memset failed");
        if (D == 128)
            chan_max_kernel<128><<<grid, kStageThreads, 0, s>>>(prm);
        else
            chan_max_kernel<64><<<grid, kStageThreads, 0, s>>>(prm);
        int e = check_launch("stage_kv_tiles (channel maxima)");
        if (e) return e;
        if (D == 128)
            chan_select_kernel<128><<<H_kv, 128, 0, s>>>(prm);
        else
            chan_select_kernel<64><<<H_kv, 64, 0, s>>>(prm);
        e = check_launch("stage_kv_tiles (channel selection)");
        if (e) return e;
    }
    if (D == 128)
        stage_tiles_kernel<128><<<grid, kStageThreads, 0, s>>>(prm);
    else
        stage_tiles_kernel<64><<<grid, kStageThreads, 0, s>>>(prm);
    return check_launch("stage_kv_tiles");
}

int skv_stage_kv_tiles(const skv_bucket* buckets, int B, int H, int S_kv, int D, int int4_group, const int32_t* rows,
                       const int32_t* counts, void* scratch, size_t scratch_bytes, void* stream) {
    return skv_stage_kv_tiles_gqa(buckets, B, H, S_kv, D, int4_group, rows, counts, nullptr, nullptr, 0, scratch,
                                  scratch_bytes, 0, stream);
}

}  // extern "C"

namespace {

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link against libcuda).
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static std::once_flag once;
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    std::call_once(once, [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
    });
    return fn;
}

template <int D>
int launch_attention(const AttnParams& prm, cudaStream_t s) {
    auto enc = tensor_map_encoder();
    if (!enc) return fail(SKV_ERR_CUDA, "attend_kv_tiles: cuTensorMapEncodeTiled is not available");
    // Q as a 2-D tensor [B*H*S_q rows, D columns] of fp16; boxes of 128 rows x 64 columns land
    // in shared memory in the 128-byte-swizzled layout the UMMA descriptors describe
    CUtensorMap qmap;
    const cuuint64_t dims[2] = {(cuuint64_t)D, (cuuint64_t)prm.B * prm.H * prm.S_q};
    const cuuint64_t strides[1] = {(cuuint64_t)D * sizeof(__half)};
    const cuuint32_t box[2] = {64, (cuuint32_t)kBM};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = enc(&qmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half*>(prm.q), dims, strides, box,
                           estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(SKV_ERR_CUDA, "attend_kv_tiles: tensor map encoding failed (%d)", (int)r);
    if (prm.pair) {
        if constexpr (D != 128) {
            return fail(SKV_ERR_UNSUPPORTED, "attend_kv_tiles: the CTA-pair pipeline needs head_dim 128");
        } else {
            // the staged tiles as rows of 128 bytes (no swizzle: they are staged in the layout the
            // MMA reads); boxes of 64 rows for K and V halves, of 16 rows for lo halves
            const size_t staged = (size_t)prm.B * prm.H_kv * prm.ntmax * staged_set_bytes(D);
            const cuuint64_t sdims[2] = {128, (cuuint64_t)(staged / 128)};
            const cuuint64_t sstr[1] = {128};
            const cuuint32_t sbox[2] = {128, 64}, lbox[2] = {128, 16};
            CUtensorMap stmap, lomap;
            CUresult r2 = enc(&stmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, prm.stage, sdims, sstr, sbox, estr,
                              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
            if (r2 == CUDA_SUCCESS)
                r2 = enc(&lomap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, prm.stage, sdims, sstr, lbox, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
            if (r2 != CUDA_SUCCESS)
                return fail(SKV_ERR_CUDA, "attend_kv_tiles: staged-tile tensor map encoding failed (%d)", (int)r2);
            const int smem = prm.n_peers > 0 ? PairLayout<true>::kAlloc : PairLayout<false>::kAlloc;
            void* kern = prm.n_peers > 0 ? reinterpret_cast<void*>(packed_attention_pair_kernel<true>)
                                         : reinterpret_cast<void*>(packed_attention_pair_kernel<false>);
            cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
            AttnParams a = prm;
            void* args[] = {&qmap, &stmap, &lomap, &a};
            const unsigned grid = (unsigned)(prm.slots & ~1);     // whole pairs (the kernel is clustered by 2)
            const cudaError_t e = cudaLaunchKernel(kern, dim3(grid > 0 ? grid : 2), dim3(kPairThreads), args,
                                                   (size_t)smem, s);
            if (e != cudaSuccess) return fail(SKV_ERR_CUDA, "attend_kv_tiles: pair launch failed: %s", cudaGetErrorString(e));
            return check_launch("attend_kv_tiles");
        }
    }
    if (cudaMemsetAsync(prm.part_flag, 0, (size_t)prm.slots * sizeof(int), s) != cudaSuccess)
        return fail(SKV_ERR_CUDA, "attend_kv_tiles: memset failed");
    int smem, threads;
    void* kern;
    if (!prm.one_tile) {
        smem = prm.n_peers > 0 ? AttnLayout<D, true>::kAlloc : AttnLayout<D, false>::kAlloc;
        if (prm.emu)
            kern = prm.n_peers > 0 ? reinterpret_cast<void*>(packed_attention_kernel<D, true, true>)
                                   : reinterpret_cast<void*>(packed_attention_kernel<D, false, true>);
        else
            kern = prm.n_peers > 0 ? reinterpret_cast<void*>(packed_attention_kernel<D, true, false>)
                                   : reinterpret_cast<void*>(packed_attention_kernel<D, false, false>);
        threads = kAttnThreads;
    } else {
        smem = prm.n_peers > 0 ? Attn1TLayout<D, true>::kAlloc : Attn1TLayout<D, false>::kAlloc;
        kern = prm.n_peers > 0 ? reinterpret_cast<void*>(packed_attention_1t_kernel<D, true>)
                               : reinterpret_cast<void*>(packed_attention_1t_kernel<D, false>);
        threads = k1TThreads;
    }
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    AttnParams a = prm;
    void* args[] = {&qmap, &a};
    const cudaError_t e = cudaLaunchCooperativeKernel(kern, dim3((unsigned)prm.slots), dim3(threads), args,
                                                      (size_t)smem, s);
    if (e != cudaSuccess)
        return fail(SKV_ERR_CUDA, "attend_kv_tiles: cooperative launch failed: %s", cudaGetErrorString(e));
    return check_launch("attend_kv_tiles");
}

}  // namespace

extern "C" {

int skv_attend_kv_tiles_peers(const void* q, int B, int H_q, int S_q, int D, int H_kv, int S_kv, const int32_t* rows,
                              const int32_t* counts, int S_new, float scale, const void* scratch,
                              size_t scratch_bytes, float* const* out_peers, int n_peers, int head_offset,
                              int H_out, int32_t* error_flag, int max_ctas, int flags, void* stream) {
    if (!q || !out_peers || !error_flag || n_peers <= 0)
        return fail(SKV_ERR_INVALID_ARGUMENT, "attend_kv_tiles_peers: null pointer or no peers");
    if (n_peers > 64 || head_offset < 0 || H_out < head_offset + H_q)
        return fail(SKV_ERR_SHAPE, "attend_kv_tiles_peers: heads %d at %d of %d, %d peers", H_q, head_offset, H_out,
                    n_peers);
    AttnParams prm;
    const float* staged = S_new > 0 ? reinterpret_cast<const float*>(scratch) : nullptr;
    // `out` is not used with peers; a non-null placeholder passes the shared checks
    float* placeholder = reinterpret_cast<float*>(const_cast<void*>(scratch));
    const int st = attn_params(q, B, H_q, S_q, D, nullptr, H_kv, S_kv, 0, rows, counts, staged, staged, S_new, scale,
                               const_cast<void*>(scratch), scratch_bytes, placeholder, error_flag, prm,
                               "attend_kv_tiles_peers", max_ctas, out_peers, n_peers, head_offset, H_out, flags);
    if (st != SKV_OK) return st;
    cudaStream_t s = as_stream(stream);
    if (cudaMemsetAsync(error_flag, 0, sizeof(int32_t), s) != cudaSuccess)
        return fail(SKV_ERR_CUDA, "attend_kv_tiles_peers: memset failed");
    return D == 128 ? launch_attention<128>(prm, s) : launch_attention<64>(prm, s);
}

int skv_attend_kv_tiles_gqa(const void* q, int B, int H_q, int S_q, int D, int H_kv, int S_kv, const int32_t* rows,
                            const int32_t* counts, int S_new, float scale, const void* scratch, size_t scratch_bytes,
                            float* out, int32_t* error_flag, int max_ctas, int flags, void* stream) {
    if (!q || !out || !error_flag) return fail(SKV_ERR_INVALID_ARGUMENT, "attend_kv_tiles: null pointer");
    AttnParams prm;
    // the dense rows are already staged: only their count matters here (a non-null placeholder
    // passes the argument checks and is never read)
    const float* staged = S_new > 0 ? reinterpret_cast<const float*>(scratch) : nullptr;
    const int st = attn_params(q, B, H_q, S_q, D, nullptr, H_kv, S_kv, 0, rows, counts, staged, staged, S_new, scale,
                               const_cast<void*>(scratch), scratch_bytes, out, error_flag, prm, "attend_kv_tiles",
                               max_ctas, nullptr, 0, 0, 0, flags);
    if (st != SKV_OK) return st;
    cudaStream_t s = as_stream(stream);
    if (cudaMemsetAsync(error_flag, 0, sizeof(int32_t), s) != cudaSuccess)
        return fail(SKV_ERR_CUDA, "attend_kv_tiles: memset failed");
    return D == 128 ? launch_attention<128>(prm, s) : launch_attention<64>(prm, s);
}

int skv_attend_kv_tiles(const void* q, int B, int H, int S_q, int D, int S_kv, const int32_t* rows,
                        const int32_t* counts, float scale, const void* scratch, size_t scratch_bytes, float* out,
                        int32_t* error_flag, void* stream) {
    return skv_attend_kv_tiles_gqa(q, B, H, S_q, D, H, S_kv, rows, counts, 0, scale, scratch, scratch_bytes, out,
                                   error_flag, 0, 0, stream);
}

int skv_packed_attention_gqa(const void* q, int B, int H_q, int S_q, int D, const skv_bucket* buckets, int H_kv,
                             int S_kv, int int4_group, const int32_t* rows, const int32_t* counts,
                             const float* k_new, const float* v_new, int S_new, float scale, void* scratch,
                             size_t scratch_bytes, float* out, int32_t* error_flag, int max_ctas, int flags,
                             void* stream) {
    if (!q || !buckets || !out || !error_flag) return fail(SKV_ERR_INVALID_ARGUMENT, "packed_attention: null pointer");
    if (H_kv <= 0 || H_q % H_kv) return fail(SKV_ERR_SHAPE, "packed_attention: %d query heads over %d KV heads", H_q, H_kv);
    const int st = skv_stage_kv_tiles_gqa(buckets, B, H_kv, S_kv, D, int4_group, rows, counts, k_new, v_new, S_new,
                                          scratch, scratch_bytes, flags, stream);
    if (st != SKV_OK) return st;
    return skv_attend_kv_tiles_gqa(q, B, H_q, S_q, D, H_kv, S_kv, rows, counts, S_new, scale, scratch, scratch_bytes,
                                   out, error_flag, max_ctas, flags, stream);
}

int skv_packed_attention(const void* q, int B, int H, int S_q, int D, const skv_bucket* buckets, int S_kv,
                         int int4_group, const int32_t* rows, const int32_t* counts, float scale, void* scratch,
                         size_t scratch_bytes, float* out, int32_t* error_flag, void* stream) {
    return skv_packed_attention_gqa(q, B, H, S_q, D, buckets, H, S_kv, int4_group, rows, counts, nullptr, nullptr, 0,
                                    scale, scratch, scratch_bytes, out, error_flag, 0, 0, stream);
}

}  // extern "C"
