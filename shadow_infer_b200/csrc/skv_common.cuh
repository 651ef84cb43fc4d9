// Shared helpers of the ShadowKV sm_100a kernels: status handling, stream
// casts, bucket geometry and warp utilities.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "shadowkv_b200.h"

namespace skv {

constexpr int kWarp = 32;
constexpr int kNumBuckets = 4;   // fp32, fp16, int8, int4
constexpr int kCodeEvicted = 4;

// Records a message in the thread-local last-error slot and returns `status`.
int fail(int status, const char* fmt, ...);
// Checks the last launch on the calling thread; SKV_OK or SKV_ERR_CUDA.
int check_launch(const char* what);

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// Number of SMs of the current device (cached per device).
int sm_count();

// Effective int4 group of packed_kv_cache.py:307.
__host__ __device__ inline int int4_group(int D, int group_size) {
    return (group_size > 0 && D % group_size == 0) ? group_size : D;
}

// Bytes of one int4 entry row: ceil(B*D/2).
__host__ __device__ inline int64_t int4_row_bytes(int B, int D) {
    return ((int64_t)B * D + 1) / 2;
}

__host__ __device__ inline int slot_code(int32_t s) { return s & 3; }
__host__ __device__ inline int32_t slot_pos(int32_t s) { return s >> 2; }
__host__ __device__ inline int32_t make_slot(int32_t pos, int code) { return (pos << 2) | code; }

__device__ __forceinline__ float warp_max(float x) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, o));
    return x;
}

// Max over aligned groups of `width` lanes (width a power of two <= 32).
__device__ __forceinline__ float group_max(float x, int width) {
    for (int o = width >> 1; o > 0; o >>= 1) x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, o));
    return x;
}

// Order-preserving 32-bit image of a float score for radix selection: ascending images are
// ascending scores (the order a stable float sort uses), -0.0 ties with +0.0, NaN sorts last.
__device__ __forceinline__ uint32_t score_bits(float f) {
    if (f != f) return 0xFFFFFFFFu;
    if (f == 0.0f) f = 0.0f;
    const uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Bounded grid barrier for cooperative launches (every block resident).  `count` only grows
// within a launch (zeroed before it): barrier number `epoch` completes when it reaches
// epoch * nblocks.  Returns false, and records the failure in *err, if the other blocks do
// not arrive within the limit or another block has failed.
__device__ __forceinline__ bool grid_sync_bounded(unsigned* count, int* err, unsigned nblocks, unsigned& epoch) {
    __shared__ int s_ok;
    __syncthreads();
    ++epoch;
    if (threadIdx.x == 0) {
        const unsigned target = epoch * nblocks;
        __threadfence();
        atomicAdd(count, 1u);
        volatile unsigned* cnt = count;
        int ok = 1;
        long long it = 0;
        while (*cnt < target) {
            if (++it > (1ll << 24) || *reinterpret_cast<volatile int*>(err)) {
                atomicExch(err, 1);
                ok = 0;
                break;
            }
            if (it > 256) __nanosleep(32);
        }
        __threadfence();
        s_ok = ok;
    }
    __syncthreads();
    return s_ok != 0;
}

__device__ __forceinline__ long long warp_sum_ll(long long x) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
    return x;
}

// IEEE round-to-nearest-even quantisers matching torch CPU
// (true division, torch.round == rint, clamp, cast).
__device__ __forceinline__ float quant_scale(float amax, float qmax) {
    float s = __fdiv_rn(amax, qmax);
    return s == 0.0f ? 1.0f : s;
}
__device__ __forceinline__ int quant_value(float x, float scale, int lo, int hi) {
    float q = rintf(__fdiv_rn(x, scale));
    q = fminf(fmaxf(q, (float)lo), (float)hi);
    return (int)q;
}

// Same result as quant_value without a division per element.  `rcp` must be
// __frcp_rn(scale).  y = x*rcp differs from the correctly rounded quotient
// fl(x/scale) by at most ~2.3e-5 for |x/scale| <= 128 (two roundings of 2^-24
// relative each, plus the half-ulp of fl itself), so rint(y) == rint(fl(x/scale))
// unless y lies within 1e-4 of a half-integer (or is not finite); only those
// rare elements take the exact IEEE division.
__device__ __forceinline__ int quant_value_fast(float x, float scale, float rcp, int lo, int hi) {
    const float y = __fmul_rn(x, rcp);
    float q = rintf(y);
    if (!(fabsf(y - q) < 0.4999f)) q = rintf(__fdiv_rn(x, scale));
    q = fminf(fmaxf(q, (float)lo), (float)hi);
    return (int)q;
}

// Copies `bytes` bytes with a warp, using 16-byte vectors when both ends allow.
__device__ __forceinline__ void warp_copy(void* dst, const void* src, int64_t bytes, int lane) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(src);
    if ((a & 15) == 0 && (bytes & 15) == 0) {
        uint4* d = reinterpret_cast<uint4*>(dst);
        const uint4* s = reinterpret_cast<const uint4*>(src);
        for (int64_t i = lane; i < bytes / 16; i += kWarp) d[i] = s[i];
    } else if ((a & 3) == 0 && (bytes & 3) == 0) {
        uint32_t* d = reinterpret_cast<uint32_t*>(dst);
        const uint32_t* s = reinterpret_cast<const uint32_t*>(src);
        for (int64_t i = lane; i < bytes / 4; i += kWarp) d[i] = s[i];
    } else {
        uint8_t* d = reinterpret_cast<uint8_t*>(dst);
        const uint8_t* s = reinterpret_cast<const uint8_t*>(src);
        for (int64_t i = lane; i < bytes; i += kWarp) d[i] = s[i];
    }
}

// Bytes per entry row (all B batches) of the K (or V) payload of bucket p.
__host__ __device__ inline int64_t payload_row_bytes(int p, int B, int D) {
    switch (p) {
        case 0: return (int64_t)B * D * 4;
        case 1: return (int64_t)B * D * 2;
        case 2: return (int64_t)B * D;
        default: return int4_row_bytes(B, D);
    }
}
// Scale floats per entry of bucket p (0 for fp32/fp16).
__host__ __device__ inline int64_t scale_row_floats(int p, int B, int D, int G) {
    return p == 2 ? (int64_t)B : (p == 3 ? (int64_t)B * G : 0);
}

// Plain-old-data copy of the 4 buckets, passed by value to kernels.
struct Buckets {
    skv_bucket b[kNumBuckets];
};

}  // namespace skv
