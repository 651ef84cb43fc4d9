// Packed attention over a CTA pair (included by attention.cu; SKV_ATTN_PAIR, head_dim 128).
//
// A cluster of two CTAs takes a unit of 256 queries of one head; CTA r (its rank in the pair)
// owns query rows r*128 .. r*128+127 of the unit, one 128-row tile.  The MMAs are tcgen05
// cta_group::2 with M = 256, issued for both CTAs by one thread of CTA 0:
//   S = Q K^T   each CTA's Q tile, and 64 of the KV tile's 128 keys from each CTA's shared
//               memory (each CTA loads half of every staged K tile and of its lo tile);
//   O += P V    each CTA's P from its own TMEM, and 64 of the 128 head dims from each CTA (each
//               CTA loads one of the two 64-dim atoms of every staged V tile).
// So a staged tile still crosses L2 -> shared memory once per 256 queries, as in the two-tile
// kernel, but a CTA holds ONE query tile: its TMEM has room for two S buffers and two O
// buffers, S runs two KV steps ahead of P V (the tensor cores never wait for the softmax of the
// step they are about to feed), and the tile's softmax is split over all eight softmax warps --
// two per TMEM lane quarter, one per column half, exchanging the row max through shared memory.
//
// Warps per CTA: 0-7 softmax (warp w: lane quarter w & 3, columns (w >> 2) * 64 .. +63),
// 8 loader, 9 MMA issuer in CTA 0 (CTA 1's warp 9 only allocates).  Both warps 9 allocate the
// pair's TMEM.  TMEM per CTA: S_0 | S_1 | O_0 | O_1 (4 x 128 columns); P(g) over the first 64
// columns of S_{g&1}; O buffers alternate by unit, so one unit's epilogue overlaps the next
// unit's MMAs.  K, V and the lo tiles come in by TMA (the staged tiles seen as rows of 128 bytes,
// no swizzle: they are staged in the swizzled layout already), each CTA's loads counted on CTA
// 0's barriers (cta_group::2 form, no multicast).  Work: whole units round-robin over the pairs.
// Every wait is bounded; after a failure a role skips its remaining work and all roles reach the
// final cluster barrier before TMEM is released.  CTA 0's loader first waits (bounded) for the
// last copies issued into every K and V stage: its barriers count both CTAs' bytes.

constexpr int kPairThreads = 10 * 32;
constexpr int kPairNK = 3;                 // K (+ lo) stages
constexpr int kPairNV = 3;                 // V stages
constexpr int kPairHalf = 16384;           // half of a staged K or V tile (D = 128)
constexpr int kPairLoHalf = kLoTile / 2;   // half of a lo tile: 64 rows x 32 bytes

template <bool PEERS>
struct PairLayout {
    static constexpr int kQ = 0;                              // 2 buffers x (128 rows x 256 B)
    static constexpr int kK = 2 * 32768;                      // kPairNK x (2 atoms x 64 rows x 128 B)
    static constexpr int kV = kK + kPairNK * kPairHalf;       // kPairNV x (128 keys x 128 B, one atom)
    static constexpr int kKc = kV + kPairNV * kPairHalf;      // kPairNK x (64 rows x 32 B)
    static constexpr int kQc = kKc + kPairNK * kPairLoHalf;   // 2 buffers x (128 rows x 32 B)
    static constexpr int kMx = kQc + 2 * kLoTile;             // [2][4][2][32] row maxes
    static constexpr int kLx = kMx + 2 * 4 * 2 * 32 * 4;      // [4][2][32] row sums
    static constexpr int kBar = kLx + 4 * 2 * 32 * 4;
    static constexpr int kNumBars = 32;
    static constexpr int kSch = kBar + kNumBars * 8;
    static constexpr int kTmemSlot = (kSch + kSchedSmemBytes + 15) / 16 * 16;
    static constexpr int kBytes = kTmemSlot + 16;
    static constexpr int kAlloc = kBytes + 1024;
    static_assert(kAlloc <= 227 * 1024, "pair attention shared memory beyond the per-CTA limit");
    static_assert((kKc % 1024) == 0 && (kQc % 1024) == 0, "swizzled tiles need 1 KB alignment");
};

__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// Bounded wait for a phase completed by arrivals from the other CTA (acquire at cluster scope).
__device__ __forceinline__ bool mbar_wait_pair(uint64_t* bar, uint32_t parity, int* err, int code,
                                               uint64_t limit_ns = 1000000000ull) {
    uint64_t t0 = 0;
    for (;;) {
        if (mbar_try_wait_cluster(bar, parity, 20000u)) return true;
        if (*reinterpret_cast<volatile int*>(err) != 0) return false;
        const uint64_t now = globaltimer_ns();
        if (t0 == 0) t0 = now;
        else if (now - t0 > limit_ns) {
            atomicCAS(err, 0, code);
            return false;
        }
    }
}

// The KV steps of a pair's units in order: units pi, pi + P, pi + 2P, ... (k = how many units of
// this pair came before), each unit one step per KV tile of its head.
struct PairCursor {
    const SchedSmem* c;
    long long u, U, stride;
    int b, h, qp, nt, j, k;
    bool valid;

    __device__ void load_unit() {
        valid = u < U;
        if (valid) Schedule::unit_start(c, u, b, h, qp, nt);
        j = 0;
    }
    __device__ void start(const SchedSmem* c_, long long first, long long stride_, long long U_) {
        c = c_;
        u = first;
        stride = stride_;
        U = U_;
        k = 0;
        load_unit();
    }
    __device__ void next() {
        if (!valid) return;
        if (++j < nt) return;
        u += stride;
        ++k;
        load_unit();
    }
    __device__ bool first() const { return j == 0; }
    __device__ bool last() const { return j == nt - 1; }
};

// Four consecutive output values at element idx (a multiple of 4): fp32, or fp16 with out_half.
__device__ __forceinline__ void pair_put4(const AttnParams& p, float* base, int64_t idx, float4 v) {
    if (p.out_half) {
        const uint2 h = make_uint2(half2_bits(__floats2half2_rn(v.x, v.y)), half2_bits(__floats2half2_rn(v.z, v.w)));
        *reinterpret_cast<uint2*>(reinterpret_cast<__half*>(base) + idx) = h;
    } else {
        *reinterpret_cast<float4*>(base + idx) = v;
    }
}
template <bool PEERS>
__device__ __forceinline__ void pair_store4(const AttnParams& p, int64_t idx, float4 v) {
    if constexpr (PEERS) {
        for (int i = 0; i < p.n_peers; ++i) pair_put4(p, p.peers[i], idx, v);
    } else {
        pair_put4(p, p.out, idx, v);
    }
}

template <bool PEERS>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kPairThreads, 1)
    packed_attention_pair_kernel(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap stmap,
                                 const __grid_constant__ CUtensorMap lomap, const __grid_constant__ AttnParams p) {
    constexpr int D = 128;
    using L = PairLayout<PEERS>;
    constexpr uint32_t TB = staged_tile_bytes(D);
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_rank();

    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBar);
    uint64_t* q_full = bars;           // [2] this CTA's Q tile landed (local TMA)
    uint64_t* q_ready = bars + 2;      // [2] CTA 0: both CTAs' Q (and Q_c) in place, one arrival each
    uint64_t* q_empty = bars + 4;      // [2] the unit's last S MMAs done (commit to both CTAs)
    uint64_t* k_full = bars + 6;       // [kPairNK] CTA 0: both halves of K (+ lo) landed (TMA bytes)
    uint64_t* k_empty = bars + 9;      // [kPairNK] the stage's S MMAs done (commit to both CTAs)
    uint64_t* v_full = bars + 12;      // [kPairNV] CTA 0: both halves of V landed
    uint64_t* v_empty = bars + 15;     // [kPairNV] the stage's P V MMAs done
    uint64_t* s_full = bars + 18;      // [2] S buffer ready (commit to both CTAs)
    uint64_t* p_full = bars + 20;      // [2] CTA 0: P of the buffer in TMEM, 16 softmax warps
    uint64_t* pv_done = bars + 22;     // every P V done (commit to both CTAs), for O rescales
    uint64_t* o_full = bars + 23;      // [2] the unit's last P V done
    uint64_t* o_empty = bars + 25;     // [2] CTA 0: O buffer read out, 16 softmax warps
    uint64_t* drain = bars + 27;       // CTA 0: every MMA done before TMEM release
    SchedSmem* ss = reinterpret_cast<SchedSmem*>(smem + L::kSch);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kTmemSlot);

    if (threadIdx.x == 0) {
        for (int i = 0; i < 2; ++i) {
            mbar_init(&q_full[i], 1);
            mbar_init(&q_ready[i], 2);
            mbar_init(&q_empty[i], 1);
            mbar_init(&s_full[i], 1);
            mbar_init(&p_full[i], 16);
            mbar_init(&o_full[i], 1);
            mbar_init(&o_empty[i], 16);
        }
        for (int i = 0; i < kPairNK; ++i) {
            mbar_init(&k_full[i], 1);
            mbar_init(&k_empty[i], 1);
        }
        for (int i = 0; i < kPairNV; ++i) {
            mbar_init(&v_full[i], 1);
            mbar_init(&v_empty[i], 1);
        }
        mbar_init(pv_done, 1);
        mbar_init(drain, 1);
        fence_mbarrier_init();
        Schedule::setup(ss, p);
    }
    if (warp == 9) {
        tmem_alloc_pair(tmem_slot, 512);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    cluster_sync_all();     // both CTAs' barriers initialised and TMEM allocated
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const long long U = (long long)p.B * ss->QP * ss->hn[ss->H];
    const long long pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
    // shared::cluster addresses of CTA 0's barriers that both CTAs arrive on / count bytes on
    auto lead = [&](uint64_t* bar) { return cluster_addr(bar, 0); };
    auto both = [&](uint64_t* bar) {         // CTA 0 commits to the barrier in both CTAs
        umma_commit_pair(cluster_addr(bar, 0));
        umma_commit_pair(cluster_addr(bar, 1));
    };
    const int* cnts = p.counts;

    if (warp < 8) {
        // ------------------------------------------------------------------ softmax
        const int qw = warp & 3, hc = warp >> 2;
        const uint32_t lane_off = (uint32_t)(qw * 32) << 16;
        float* mx = reinterpret_cast<float*>(smem + L::kMx);
        float* lx = reinterpret_cast<float*>(smem + L::kLx);
        const float sl2 = p.scale_log2;
        PairCursor cur;
        cur.start(ss, pair, npairs, U);
        long long g = 0;
        bool ok = true;
        float m_ref = -INFINITY, l = 0.0f;
        int n_stored = 0;
        for (; cur.valid; cur.next(), ++g) {
            const int b = (int)(g & 1);
            if (cur.first()) {
                const int* cn = cnts + (int64_t)(cur.h / p.rep) * 5;
                n_stored = cn[0] + cn[1] + cn[2] + cn[3] + p.S_new;
                const int n_ev = cn[4];
                m_ref = n_ev > 0 ? 0.0f : -INFINITY;     // evicted rows: logit 0, counted once (half 0)
                l = (hc == 0) ? (float)n_ev : 0.0f;
            }
            if (ok) ok = warp_wait(&s_full[b], (uint32_t)((g >> 1) & 1), p.err, kErrSFull);
            uint32_t sc[64];
            float pm = -INFINITY;
            const uint32_t tS = tmem + b * 128 + hc * 64 + lane_off;
            if (ok) {
                tc_fence_after();
                tmem_ld32(tS, *reinterpret_cast<uint32_t(*)[32]>(&sc[0]));
                tmem_ld32(tS + 32, *reinterpret_cast<uint32_t(*)[32]>(&sc[32]));
                tmem_wait_ld();
                const int n_valid = n_stored - cur.j * kBN - hc * 64;
                if (n_valid < 64) {
#pragma unroll
                    for (int c = 0; c < 64; ++c)
                        if (c >= n_valid) sc[c] = __float_as_uint(-INFINITY);
                }
                pm = row_max<64>(sc);
            }
            // the two column halves of a row meet every step, also after a failure; past this
            // barrier both halves' S loads are done, so P may go over S's first 64 columns
            mx[((b * 4 + qw) * 2 + hc) * 32 + lane] = pm;
            tc_fence_before();
            named_bar_sync(1 + qw, 64);
            tc_fence_after();
            const float mt = fmaxf(pm, mx[((b * 4 + qw) * 2 + (hc ^ 1)) * 32 + lane]) * sl2;
            if (ok) {
                const bool need = mt > m_ref + kRescaleThreshold;
                const bool rescale = __any_sync(0xffffffffu, need);
                const float fac = need ? ex2(m_ref - mt) : 1.0f;
                if (need) m_ref = mt;
                l *= fac;
                const float2 sl2x2 = make_float2(sl2, sl2), negm2 = make_float2(-m_ref, -m_ref);
                float2 acc0 = make_float2(0.f, 0.f), acc1 = make_float2(0.f, 0.f);
#pragma unroll
                for (int c = 0; c < 2; ++c) {
                    uint32_t pk[16];
#pragma unroll
                    for (int i = 0; i < 32; i += 2) {
                        const int col = c * 32 + i;
                        const float2 x = __ffma2_rn(
                            make_float2(__uint_as_float(sc[col]), __uint_as_float(sc[col + 1])), sl2x2, negm2);
                        const float2 e = make_float2(ex2(x.x), ex2(x.y));
                        if ((col >> 1) & 1)
                            acc1 = __fadd2_rn(acc1, e);
                        else
                            acc0 = __fadd2_rn(acc0, e);
                        pk[i / 2] = half2_bits(__floats2half2_rn(e.x, e.y));
                    }
                    // P of keys hc*64 + c*32 .. over the first half of S_b's columns
                    tmem_st16(tmem + b * 128 + hc * 32 + c * 16 + lane_off, pk);
                }
                l += (acc0.x + acc0.y) + (acc1.x + acc1.y);
                if (rescale && !cur.first()) {
                    // O holds the unit's steps so far once the previous P V is done
                    ok = warp_wait(pv_done, (uint32_t)((g - 1) & 1), p.err, kErrOFull);
                    if (ok) {
                        tc_fence_after();
                        const uint32_t tO = tmem + 256 + (cur.k & 1) * 128 + hc * 64 + lane_off;
                        uint32_t o[32];
#pragma unroll
                        for (int c = 0; c < 2; ++c) {
                            tmem_ld32(tO + c * 32, o);
                            tmem_wait_ld();
#pragma unroll
                            for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * fac);
                            tmem_st32(tO + c * 32, o);
                        }
                    }
                }
                tmem_wait_st();
                tc_fence_before();
            }
            __syncwarp();
            if (lane == 0) mbar_arrive_remote(lead(&p_full[b]));
            if (!cur.last()) continue;
            // ---------------------------------------------------------------- epilogue
            const int ob = cur.k & 1;
            if (ok) ok = warp_wait(&o_full[ob], (uint32_t)((cur.k >> 1) & 1), p.err, kErrOFull);
            lx[(qw * 2 + hc) * 32 + lane] = l;
            named_bar_sync(1 + qw, 64);
            const float lt = l + lx[(qw * 2 + (hc ^ 1)) * 32 + lane];
            if (ok) {
                tc_fence_after();
                const float inv = lt > 0.0f ? 1.0f / lt : 0.0f;
                const int row = cur.qp * kUnitRows + (int)rank * kBM + qw * 32 + lane;
                const int64_t obase = (((int64_t)cur.b * p.H_out + p.head_off + cur.h) * p.S_q + row) * D + hc * 64;
                const uint32_t tO = tmem + 256 + ob * 128 + hc * 64 + lane_off;
#pragma unroll
                for (int c = 0; c < 2; ++c) {
                    uint32_t o[32];
                    tmem_ld32(tO + c * 32, o);
                    tmem_wait_ld();
                    if (row < p.S_q) {
#pragma unroll
                        for (int i = 0; i < 32; i += 4)
                            pair_store4<PEERS>(p, obase + c * 32 + i,
                                               make_float4(__uint_as_float(o[i]) * inv, __uint_as_float(o[i + 1]) * inv,
                                                           __uint_as_float(o[i + 2]) * inv,
                                                           __uint_as_float(o[i + 3]) * inv));
                    }
                }
                tc_fence_before();
            }
            __syncwarp();
            if (lane == 0) mbar_arrive_remote(lead(&o_empty[ob]));
        }
        // units of heads without a stored entry are never scheduled: their output is zero
        const long long UA = (long long)p.B * p.H * p.QP;
        for (long long u = pair; u < UA; u += npairs) {
            const int qp = (int)(u % p.QP);
            const int hh = (int)((u / p.QP) % p.H);
            const int bb = (int)(u / ((long long)p.QP * p.H));
            if (ss->hp[hh + 1] != ss->hp[hh]) continue;
            const int row = qp * kUnitRows + (int)rank * kBM + qw * 32 + lane;
            if (row >= p.S_q) continue;
            const int64_t ob = (((int64_t)bb * p.H_out + p.head_off + hh) * p.S_q + row) * D + hc * 64;
            for (int i = 0; i < 64; i += 4) pair_store4<PEERS>(p, ob + i, make_float4(0.f, 0.f, 0.f, 0.f));
        }
    } else if (warp == 8) {
        // ------------------------------------------------------------------ loader
        // K (+ lo) of step g + 2 and V of step g per iteration, in the order the MMAs need
        // them; a unit's Q tile (and the Q_c gather) before its first K.
        PairCursor kc, vc;
        kc.start(ss, pair, npairs, U);
        vc.start(ss, pair, npairs, U);
        long long gk = 0, gv = 0;
        long long k_issued = 0, v_issued = 0;     // K and V steps whose copies this CTA issued
        bool ok = true;
        HeadRows hr;      // the head of cursor kc's unit
        auto load_q = [&](const PairCursor& c) -> bool {
            const int qb = c.k & 1;
            if (c.k >= 2 && !warp_wait(&q_empty[qb], (uint32_t)(((c.k - 2) >> 1) & 1), p.err, kErrQEmpty))
                return false;
            const int qrow = (c.b * p.H + c.h) * p.S_q + c.qp * kUnitRows + (int)rank * kBM;
            if (lane == 0) {
                mbar_arrive_expect_tx(&q_full[qb], TB);
#pragma unroll
                for (int a = 0; a < D / 64; ++a)
                    tma_load_2d(smem + L::kQ + qb * TB + a * kBM * 128, &qmap, a * 64, qrow, &q_full[qb]);
            }
            __syncwarp();
            if (!warp_wait(&q_full[qb], (uint32_t)((c.k >> 1) & 1), p.err, kErrQFull)) return false;
            if (p.klo) {
                // Q_c: this tile's queries on the head's selected channels, 32-byte-swizzled rows
                const int selc = lane < kLoCh ? __ldg(p.sel + (int64_t)(c.h / p.rep) * kLoCh + lane) : 0;
                int sc[kLoCh];
#pragma unroll
                for (int i = 0; i < kLoCh; ++i) sc[i] = __shfl_sync(0xffffffffu, selc, i) & (D - 1);
                const uint8_t* qt = smem + L::kQ + qb * TB;
                uint8_t* qcp = smem + L::kQc + qb * kLoTile;
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
                    *reinterpret_cast<uint4*>(qcp + sw32_offset(r, 0)) = make_uint4(w[0], w[1], w[2], w[3]);
                    *reinterpret_cast<uint4*>(qcp + sw32_offset(r, 1)) = make_uint4(w[4], w[5], w[6], w[7]);
                }
                fence_proxy_async_smem();
            }
            __syncwarp();
            if (lane == 0) mbar_arrive_remote(lead(&q_ready[qb]));
            return true;
        };
        auto load_k = [&](const PairCursor& c, long long g) -> bool {
            const int s = (int)(g % kPairNK);
            const long long n = g / kPairNK;
            if (n >= 1 && !warp_wait(&k_empty[s], (uint32_t)((n - 1) & 1), p.err, kErrKEmpty)) return false;
            if (c.first()) hr.load(p, c.h);
            const bool lo = !hr.exact(c.j);
            if (lane == 0) {
                const int64_t set = staged_offset(p, c.b, c.h / p.rep, c.j, D);
                if (rank == 0) mbar_arrive_expect_tx(&k_full[s], 2 * (kPairHalf + (lo ? kPairLoHalf : 0)));
                const uint32_t bar = lead(&k_full[s]);
#pragma unroll
                for (int a = 0; a < 2; ++a)
                    tma_load_2d_pair(smem + L::kK + s * kPairHalf + a * (kPairHalf / 2), &stmap, 0,
                                     (int)((set + a * (TB / 2) + rank * (TB / 4)) / 128), bar);
                if (lo)
                    tma_load_2d_pair(smem + L::kKc + s * kPairLoHalf, &lomap, 0,
                                     (int)((set + 2 * TB + rank * kPairLoHalf) / 128), bar);
            }
            __syncwarp();
            k_issued = g + 1;
            return true;
        };
        auto load_v = [&](const PairCursor& c, long long g) -> bool {
            const int s = (int)(g % kPairNV);
            const long long n = g / kPairNV;
            if (n >= 1 && !warp_wait(&v_empty[s], (uint32_t)((n - 1) & 1), p.err, kErrVEmpty)) return false;
            if (lane == 0) {
                const int64_t set = staged_offset(p, c.b, c.h / p.rep, c.j, D);
                if (rank == 0) mbar_arrive_expect_tx(&v_full[s], 2 * kPairHalf);
                const uint32_t bar = lead(&v_full[s]);
#pragma unroll
                for (int i = 0; i < 2; ++i)
                    tma_load_2d_pair(smem + L::kV + s * kPairHalf + i * (kPairHalf / 2), &stmap, 0,
                                     (int)((set + TB + rank * kPairHalf + i * (kPairHalf / 2)) / 128), bar);
            }
            __syncwarp();
            v_issued = g + 1;
            return true;
        };
        // K of the first two steps ahead of any V
        for (int i = 0; i < 2 && ok && kc.valid; ++i, kc.next(), ++gk) {
            if (kc.first()) ok = load_q(kc);
            if (ok) ok = load_k(kc, gk);
        }
        for (; ok && vc.valid; vc.next(), ++gv) {
            if (kc.valid) {
                if (kc.first()) ok = load_q(kc);
                if (ok) ok = load_k(kc, gk);
                kc.next();
                ++gk;
            }
            if (ok) ok = load_v(vc, gv);
        }
        // every copy issued lands before the pair can exit (a no-op when the MMAs consumed them;
        // after a pipeline timeout, bounded): CTA 0's barriers count both CTAs' bytes
        if (rank == 0 && lane == 0) {
            for (long long g = k_issued - 1; g >= 0 && g >= k_issued - kPairNK; --g)
                mbar_wait_spin(&k_full[g % kPairNK], (uint32_t)((g / kPairNK) & 1), p.err, kErrCopy);
            for (long long g = v_issued - 1; g >= 0 && g >= v_issued - kPairNV; --g)
                mbar_wait_spin(&v_full[g % kPairNV], (uint32_t)((g / kPairNV) & 1), p.err, kErrCopy);
        }
        __syncwarp();
    } else if (rank == 0) {
        // ----------------------------------------------------------------- MMA issue (CTA 0)
        if (lane == 0) {
            const uint32_t idesc_s = idesc_f16_f32(256, kBN, false, false);
            const uint32_t idesc_o = idesc_f16_f32(256, D, false, true);
            const uint64_t qd0 = smem_desc_sw128(smem_u32(smem + L::kQ), 16, 1024);
            const uint64_t kd0 = smem_desc_sw128(smem_u32(smem + L::kK), 16, 1024);
            const uint64_t vd0 = smem_desc_sw128(smem_u32(smem + L::kV), kBN * 128, 1024);
            const uint64_t qcd0 = smem_desc_sw32(smem_u32(smem + L::kQc), 16, 256);
            const uint64_t kcd0 = smem_desc_sw32(smem_u32(smem + L::kKc), 16, 256);
            PairCursor pc, sc;
            pc.start(ss, pair, npairs, U);
            sc.start(ss, pair, npairs, U);
            long long g = 0, gs = 0;
            bool ok = true, issued = false;
            HeadRows hr;      // the head of cursor sc's unit (global loads once per unit, off the step loop)
            // S of step gs (cursor sc) into S buffer gs & 1
            auto issue_s = [&]() -> bool {
                const int ks = (int)(gs % kPairNK);
                const int qb = sc.k & 1;
                if (sc.first()) hr.load(p, sc.h);
                if ((sc.first() && !mbar_wait_pair(&q_ready[qb], (uint32_t)((sc.k >> 1) & 1), p.err, kErrQFull)) ||
                    !mbar_wait_spin(&k_full[ks], (uint32_t)((gs / kPairNK) & 1), p.err, kErrKFull))
                    return false;
                tc_fence_after();
                const uint32_t d = tmem + (uint32_t)(gs & 1) * 128;
                const uint64_t qd = qd0 + (uint64_t)((qb * TB) >> 4);
                const uint64_t kd = kd0 + (uint64_t)((ks * kPairHalf) >> 4);
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk) {
                    const uint64_t offa = (uint64_t)((((kk >> 2) * (kBM * 128)) + (kk & 3) * 32) >> 4);
                    const uint64_t offb = (uint64_t)((((kk >> 2) * (kPairHalf / 2)) + (kk & 3) * 32) >> 4);
                    umma_pair(d, qd + offa, kd + offb, idesc_s, kk > 0 ? 1u : 0u);
                }
                if (!hr.exact(sc.j))
                    umma_pair(d, qcd0 + (uint64_t)((qb * kLoTile) >> 4), kcd0 + (uint64_t)((ks * kPairLoHalf) >> 4),
                              idesc_s, 1u);
                both(&s_full[gs & 1]);
                both(&k_empty[ks]);
                if (sc.last()) both(&q_empty[qb]);
                issued = true;
                sc.next();
                ++gs;
                return true;
            };
            for (int i = 0; i < 2 && ok && sc.valid; ++i) ok = issue_s();
            for (; ok && pc.valid; pc.next(), ++g) {
                const int b = (int)(g & 1);
                const int vs = (int)(g % kPairNV);
                const int ob = pc.k & 1;
                if (!mbar_wait_pair(&p_full[b], (uint32_t)((g >> 1) & 1), p.err, kErrPFull) ||
                    !mbar_wait_spin(&v_full[vs], (uint32_t)((g / kPairNV) & 1), p.err, kErrVFull) ||
                    (pc.first() && pc.k >= 2 &&
                     !mbar_wait_pair(&o_empty[ob], (uint32_t)(((pc.k - 2) >> 1) & 1), p.err, kErrOEmpty))) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d = tmem + 256 + ob * 128, a = tmem + b * 128;
                const uint64_t vd = vd0 + (uint64_t)((vs * kPairHalf) >> 4);
#pragma unroll
                for (int kk = 0; kk < kBN / 16; ++kk)
                    umma_pair_ts(d, a + kk * 8, vd + (uint64_t)((kk * 16 * 128) >> 4), idesc_o,
                                 (!pc.first() || kk > 0) ? 1u : 0u);
                both(&v_empty[vs]);
                both(pv_done);
                if (pc.last()) both(&o_full[ob]);
                // S two steps ahead reuses buffer b, whose P this P V has read (the pipe runs in order)
                if (sc.valid) ok = issue_s();
            }
            if (issued) {
                umma_commit_pair(cluster_addr(drain, 0));
                mbar_wait_spin(drain, 0, p.err, kErrDrain);
            }
        }
        __syncwarp();
    }

    tc_fence_before();
    cluster_sync_all();     // every MMA into both CTAs' TMEM has completed, every remote arrival landed
    if (warp == 9) {
        tc_fence_after();
        tmem_dealloc_pair(tmem, 512);
    }
}
