// Packed attention, single-query-tile pipeline (included by attention.cu; opt-in with
// SKV_ATTN_ONE_TILE).  Measured against the two-tile kernel it is slower on long sequences --
// every staged K/V tile now serves 128 queries instead of 256, which doubles the L2 -> shared
// memory traffic (~7 TB/s at the measured limit) -- and slightly faster on short query blocks
// (more, smaller work units).
//
// One work unit = 128 queries of one head.  TMEM holds two score buffers and the output:
// S[0] | S[1] | O (128 + 128 + D columns), so the scores of KV step j+1 are computed while the
// softmax of step j runs, and the per-step chain is softmax(j) -> P(j) V(j) -> S(j+2) instead
// of S -> softmax -> P V on one buffer.  Warps:
//   0-3  softmax (thread = query row = TMEM lane; warp w reads lane quarter w), then the
//        epilogue of the unit (the same merge / peer-store paths as the two-tile kernel);
//   4    loader: Q (double-buffered by segment, TMA 128B swizzle, no multicast), the Q_c gather
//        for the lo correction, K (+ lo tile) and V rings of two stages;
//   5    MMA issuer: S(g) = Q K(g)^T (+ Q_c K_lo(g)^T) into S[g & 1], P(g) V(g) into O, issued in
//        the order S(0), S(1), PV(0), S(2), PV(1), S(3), ... (a buffer is rewritten only after the
//        P V that reads it, and the tensor pipe runs in issue order).
// Every wait is bounded (the error word records the first timeout; all roles then drain).

constexpr int k1TSoftmaxWarps = 4;
constexpr int k1TLoadWarp = 4;
constexpr int k1TMmaWarp = 5;
constexpr int k1TThreads = 6 * 32;
constexpr int k1TUnitRows = kBM;   // queries per work unit

template <int D, bool PEERS = false>
struct Attn1TLayout {
    static constexpr int NA = D / 64;
    static constexpr int kTile = staged_tile_bytes(D);
    static constexpr int kQ = 0;                        // two Q buffers (segment parity)
    static constexpr int kK = kQ + 2 * kTile;           // two K stages
    static constexpr int kV = kK + 2 * kTile;           // two V stages
    static constexpr int kQc = kV + 2 * kTile;          // two Q_c buffers (segment parity)
    static constexpr int kKc = kQc + 2 * kLoTile;       // two K lo stages
    static constexpr int kBar = kKc + 2 * kLoTile;
    static constexpr int kNumBars = 24;
    static constexpr int kSch = kBar + kNumBars * 8;
    static constexpr int kOut = (kSch + kSchedSmemBytes + 127) / 128 * 128;
    static constexpr int kOutRows = 4;
    static constexpr int kMisc = kOut + (PEERS ? k1TSoftmaxWarps * kOutRows * D * 4 : 0);
    static constexpr int kTmemSlot = kMisc + 16;
    static constexpr int kBytes = kTmemSlot + 16;
    static constexpr int kAlloc = (kBytes + 1024) > 120 * 1024 ? (kBytes + 1024) : 120 * 1024;
    static_assert(kAlloc <= 227 * 1024, "attention shared memory beyond the per-CTA limit");
};

// A cursor over the KV steps of this CTA's segments (the MMA warp keeps two: S runs two steps
// ahead of P V).
struct StepCursor {
    Schedule sch;
    Segment sg;
    HeadRows hr;
    int j = 0, si = -1;
    long long g = 0;
    bool valid = false;
    __device__ void start(const Schedule& s, const AttnParams& p) {
        sch = s;
        valid = sch.next(sg);
        if (valid) {
            j = sg.j0;
            si = 0;
            hr.load(p, sg.h);
        }
    }
    __device__ void advance(const AttnParams& p) {
        ++g;
        if (++j < sg.j1) return;
        valid = sch.next(sg);
        if (valid) {
            j = sg.j0;
            ++si;
            hr.load(p, sg.h);
        }
    }
    __device__ bool first() const { return j == sg.j0; }
    __device__ bool last() const { return j + 1 == sg.j1; }
};

template <int D, bool PEERS>
__global__ void __launch_bounds__(k1TThreads, 1)
    packed_attention_1t_kernel(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ AttnParams p) {
    using L = Attn1TLayout<D, PEERS>;
    constexpr int NA = L::NA;
    constexpr uint32_t TB = L::kTile;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBar);
    uint64_t* q_full = bars + 0;        // [2] per Q buffer: expect_tx arrive + TMA bytes
    uint64_t* q_empty = bars + 2;       // [2] per Q buffer: commit after the segment's last S MMAs
    uint64_t* qc_full = bars + 4;       // [2] per Q buffer: loader warp, Q_c gathered
    uint64_t* k_full = bars + 6;        // [2] ring stages (K tile + lo tile)
    uint64_t* k_empty = bars + 8;       // [2] commit
    uint64_t* v_full = bars + 10;       // [2]
    uint64_t* v_empty = bars + 12;      // [2] commit
    uint64_t* s_full = bars + 14;       // [2] per score buffer, commit
    uint64_t* p_full = bars + 16;       // [2] per score buffer, 4 softmax warps
    uint64_t* o_full = bars + 18;       // commit after the segment's last P V
    uint64_t* o_empty = bars + 19;      // 4 softmax warps: O read out
    uint64_t* pv_done = bars + 20;      // commit after every P V (an O rescale waits for it)
    uint64_t* drain = bars + 21;        // commit, drain before TMEM release
    SchedSmem* ss = reinterpret_cast<SchedSmem*>(smem + L::kSch);
    const int* hp = ss->hp;
    int* misc = reinterpret_cast<int*>(smem + L::kMisc);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kTmemSlot);

    if (threadIdx.x == 0) {
        for (int s = 0; s < 2; ++s) {
            mbar_init(&q_full[s], 1);
            mbar_init(&q_empty[s], 1);
            mbar_init(&qc_full[s], 1);
            mbar_init(&k_full[s], 1);
            mbar_init(&k_empty[s], 1);
            mbar_init(&v_full[s], 1);
            mbar_init(&v_empty[s], 1);
            mbar_init(&s_full[s], 1);
            mbar_init(&p_full[s], k1TSoftmaxWarps);
        }
        mbar_init(o_full, 1);
        mbar_init(o_empty, k1TSoftmaxWarps);
        mbar_init(pv_done, 1);
        mbar_init(drain, 1);
        fence_mbarrier_init();
        Schedule::setup(ss, p);
    }
    if (warp == k1TMmaWarp) {
        tmem_alloc(tmem_slot, kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    Schedule sched;
    sched.init(ss);

    if (warp < k1TSoftmaxWarps) {
        // ------------------------------------------------------------------ softmax
        const int qw = warp;                             // TMEM lane quarter: rows qw*32 + lane
        const uint32_t lane_off = (uint32_t)(qw * 32) << 16;
        const uint32_t tO = tmem + 2 * kBN + lane_off;
        const float sl2 = p.scale_log2;
        const int rt = qw * 32;                          // first row of this warp in a unit
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
                const int sb = (int)(g & 1);                 // score buffer of this step
                const uint32_t tS = tmem + sb * kBN + lane_off;
                if (!warp_wait(&s_full[sb], (uint32_t)((g >> 1) & 1), p.err, kErrSFull)) { ok = false; break; }
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
                float mx0 = -INFINITY, mx1 = -INFINITY, mx2 = -INFINITY, mx3 = -INFINITY;
#pragma unroll
                for (int i = 0; i < kBN; i += 8) {
                    mx0 = fmax3(mx0, __uint_as_float(sc[i]), __uint_as_float(sc[i + 1]));
                    mx1 = fmax3(mx1, __uint_as_float(sc[i + 2]), __uint_as_float(sc[i + 3]));
                    mx2 = fmax3(mx2, __uint_as_float(sc[i + 4]), __uint_as_float(sc[i + 5]));
                    mx3 = fmax3(mx3, __uint_as_float(sc[i + 6]), __uint_as_float(sc[i + 7]));
                }
                const float mt = fmaxf(fmaxf(mx0, mx1), fmaxf(mx2, mx3)) * sl2;
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
                        const float2 e = make_float2(ex2(x.x), ex2(x.y));
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
                    // O holds this segment's steps so far; the previous step's P V may still be
                    // running (it was issued when that step's P was published), so wait for it,
                    // then rescale O before this step's P V (which waits for p_full) adds to it
                    if (!warp_wait(pv_done, (uint32_t)((g - 1) & 1), p.err, kErrOFull)) { ok = false; break; }
                    tc_fence_after();
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
                if (lane == 0) mbar_arrive(&p_full[sb]);
            }
            if (!ok) break;
            // ---------------------------------------------------------------- epilogue
            if (!warp_wait(o_full, (uint32_t)(si & 1), p.err, kErrOFull)) { ok = false; break; }
            tc_fence_after();
            const bool split_tail = sg.j0 > 0;                   // a later part: publish, unnormalised
            const bool split_head = first_part && sg.j1 < sg.nt; // first part: merge the later parts
            // later parts live in CTAs blockIdx.x + 1 .. + np (each publishes into its own slot)
            const int np = split_head ? sched.partners(sg) : 0;
            const int slot = blockIdx.x + 1;
            float mB = -INFINITY, lB = 0.0f;
            for (int i = 0; i < np; ++i) {
                int got = 1;
                if (lane == 0) got = wait_flag(p.part_flag + slot + i, k1TSoftmaxWarps, p.err, kErrPartial) ? 1 : 0;
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
            const int row0 = sg.qp * k1TUnitRows + rt;           // query row within the head
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
                                          o_empty, oslot);
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
                                        if (lane == 0) mbar_arrive(o_empty);
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
                            if (lane == 0) mbar_arrive(o_empty);
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
                                    if (lane == 0) mbar_arrive(o_empty);
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
                    if (lane == 0) mbar_arrive(o_empty);
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
            const int row0 = qp * k1TUnitRows + rt;
            const int64_t ob = (((int64_t)bb * p.H_out + p.head_off + hh) * p.S_q + row0) * D;
            for (int r = 0; r < min(32, p.S_q - row0); ++r)
                for (int d = 2 * lane; d < D; d += 64) out_store<PEERS>(p, ob + (int64_t)r * D + d, make_float2(0.0f, 0.0f));
        }
        if constexpr (PEERS) {
            // the staged rows' bulk stores have completed before the CTA (and its shared memory) ends
            if (lane == 0) bulk_wait0();
            __syncwarp();
        }
    } else if (warp == k1TLoadWarp) {
        // ------------------------------------------------------------------ loader
        Segment sg;
        long long g = 0;
        int si = 0, nq[2] = {0, 0};
        int nk[2] = {0, 0}, nv[2] = {0, 0};          // copies issued per stage (lane 0)
        bool ok = true;
        auto lane0_wait = [&](uint64_t* bar, uint32_t parity, int code) -> bool {
            int r = 1;
            if (lane == 0) r = mbar_wait_spin(bar, parity, p.err, code) ? 1 : 0;
            return __shfl_sync(0xffffffffu, r, 0) != 0;
        };
        while (ok && sched.next(sg)) {
            const int qb = si & 1;                   // Q buffer of this segment
            // the buffer's previous segment (si - 2) has issued its last S MMAs and they completed
            if (si >= 2 && !lane0_wait(&q_empty[qb], (uint32_t)(((si >> 1) - 1) & 1), kErrQEmpty)) break;
            const int qrow = (sg.b * p.H + sg.h) * p.S_q + sg.qp * k1TUnitRows;
            if (lane == 0) {
                mbar_arrive_expect_tx(&q_full[qb], TB);
#pragma unroll
                for (int a = 0; a < NA; ++a)
                    tma_load_2d(smem + L::kQ + qb * TB + a * kBM * 128, &qmap, a * 64, qrow, &q_full[qb]);
                ++nq[qb];
            }
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
                    // Q_c of this segment (its buffer's last reader, segment si - 2, is done: q_empty)
                    if (!warp_wait(&q_full[qb], (uint32_t)((si >> 1) & 1), p.err, kErrQFull)) {
                        ok = false;
                        break;
                    }
                    int sc[kLoCh];
#pragma unroll
                    for (int i = 0; i < kLoCh; ++i) sc[i] = __shfl_sync(0xffffffffu, selc, i) & (D - 1);  // in the tile
                    const uint8_t* qt = smem + L::kQ + qb * TB;
                    uint8_t* qc = smem + L::kQc + qb * kLoTile;
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
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&qc_full[qb]);
                }
            }
            ++si;
        }
        if (lane == 0) {
            // every copy issued lands before the CTA can exit (a no-op when the MMA consumed them)
            for (int s = 0; s < 2; ++s) {
                if (nq[s]) mbar_wait_spin(&q_full[s], (uint32_t)((nq[s] - 1) & 1), p.err, kErrCopy);
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
            const uint32_t tO = tmem + 2 * kBN;
            StepCursor cs, cp;                       // S runs two steps ahead of P V
            cs.start(sched, p);
            cp.start(sched, p);
            bool ok = true, issued = false;
            // S(g) into score buffer g & 1, from the Q buffer of its segment and K stage g & 1
            auto issue_s = [&](const StepCursor& c) -> bool {
                const int qb = c.si & 1, ks = (int)(c.g & 1);
                if (c.first()) {
                    if (!mbar_wait_spin(&q_full[qb], (uint32_t)((c.si >> 1) & 1), p.err, kErrQFull)) return false;
                    if (p.klo && !mbar_wait_spin(&qc_full[qb], (uint32_t)((c.si >> 1) & 1), p.err, kErrQFull))
                        return false;
                }
                if (!mbar_wait_spin(&k_full[ks], (uint32_t)((c.g >> 1) & 1), p.err, kErrKFull)) return false;
                tc_fence_after();
                const uint32_t q_base = smem_u32(smem + L::kQ + qb * TB);
                const uint32_t k_base = smem_u32(smem + L::kK + ks * TB);
                const uint32_t dS = tmem + (uint32_t)ks * kBN;
#pragma unroll
                for (int k = 0; k < D / 16; ++k) {
                    const uint32_t off = (k >> 2) * (kBN * 128) + (k & 3) * 32;
                    umma_f16(dS, smem_desc_sw128(q_base + off, 16, 1024), smem_desc_sw128(k_base + off, 16, 1024),
                             idesc_s, k > 0 ? 1u : 0u);
                }
                if (!c.hr.exact(c.j))
                    umma_f16(dS, smem_desc_sw32(smem_u32(smem + L::kQc + qb * kLoTile), 16, 256),
                             smem_desc_sw32(smem_u32(smem + L::kKc + ks * kLoTile), 16, 256), idesc_s, 1u);
                umma_commit(&s_full[ks]);
                umma_commit(&k_empty[ks]);
                if (c.last()) umma_commit(&q_empty[qb]);
                issued = true;
                return true;
            };
            // P(g) V(g) into O (P from score buffer g & 1, V stage g & 1)
            auto issue_pv = [&](const StepCursor& c) -> bool {
                const int vs = (int)(c.g & 1);
                if (!mbar_wait_spin(&v_full[vs], (uint32_t)((c.g >> 1) & 1), p.err, kErrVFull) ||
                    !mbar_wait_spin(&p_full[vs], (uint32_t)((c.g >> 1) & 1), p.err, kErrPFull))
                    return false;
                // the previous segment's O has been read out before this segment's first P V
                if (c.first() && c.si > 0 && !mbar_wait_spin(o_empty, (uint32_t)((c.si - 1) & 1), p.err, kErrOEmpty))
                    return false;
                tc_fence_after();
                const uint32_t v_base = smem_u32(smem + L::kV + vs * TB);
                const uint32_t tP = tmem + (uint32_t)vs * kBN;
#pragma unroll
                for (int k = 0; k < kBN / 16; ++k)
                    umma_f16_ts(tO, tP + k * 8, smem_desc_sw128(v_base + k * 16 * 128, kBN * 128, 1024), idesc_o,
                                (!c.first() || k > 0) ? 1u : 0u);
                umma_commit(pv_done);
                umma_commit(&v_empty[vs]);
                if (c.last()) umma_commit(o_full);
                return true;
            };
            if (cs.valid) {
                ok = issue_s(cs);
                cs.advance(p);
            }
            if (ok && cs.valid) {
                ok = issue_s(cs);
                cs.advance(p);
            }
            while (ok && cp.valid) {
                ok = issue_pv(cp);
                cp.advance(p);
                if (ok && cs.valid) {
                    ok = issue_s(cs);                // into the buffer the P V just issued reads
                    cs.advance(p);
                }
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
    if (warp == k1TMmaWarp) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}
