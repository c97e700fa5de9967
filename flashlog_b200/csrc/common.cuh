// common.cuh -- shared device helpers for the FlashLog B200 kernels.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>

#include "../../include/flashlog_b200.h"

namespace fl {

constexpr int kWarp = 32;
constexpr unsigned kFull = 0xffffffffu;

// ---- error state (thread-local message, set by the host entry points) ----
void set_error(const char *fmt, ...);
int check_launch(const char *what);

#define FL_REQUIRE(cond, ...)                 \
    do {                                      \
        if (!(cond)) {                        \
            ::fl::set_error(__VA_ARGS__);     \
            return FL_EINVAL;                 \
        }                                     \
    } while (0)

#define FL_CUDA(call)                                                          \
    do {                                                                       \
        cudaError_t e_ = (call);                                               \
        if (e_ != cudaSuccess) {                                               \
            ::fl::set_error("%s: %s", #call, cudaGetErrorString(e_));          \
            return FL_ECUDA;                                                   \
        }                                                                      \
    } while (0)

inline cudaStream_t as_stream(fl_stream_t s) { return reinterpret_cast<cudaStream_t>(s); }

// Every kernel of the library is launched through launch(), which counts the
// launches (fl_launch_count) so a caller can state how many of this library's
// kernels ran in a timed region.
void note_launch();

template <typename... KArgs, typename... Args>
inline void launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args &&...args) {
    note_launch();
    kernel<<<grid, block, smem, st>>>(static_cast<KArgs>(args)...);
}

// ---- dropout keep bits (fl_value_dropout and the fused forms) --------------
// SplitMix64 output function (G. Steele, D. Lea, C. Flood, "Fast splittable
// pseudorandom number generators", OOPSLA 2014): a bijective 64-bit mix.
__device__ __forceinline__ uint64_t splitmix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

// Kernel-side dropout: position i is kept iff the high 32 bits of
// splitmix64(key + i) reach cut; a kept value is scaled by `scale`, a
// dropped one multiplied by 0.  on == 0: no dropout.
struct DropoutArgs {
    uint64_t seed, subseq, cut;
    const int64_t *counter;
    float scale;
    int on;
};

// key of one launch: splitmix64(seed ^ splitmix64((*counter << 16) | subseq))
__device__ __forceinline__ uint64_t dropout_key(const DropoutArgs &d) {
    const uint64_t c = d.counter != nullptr ? static_cast<uint64_t>(*d.counter) : 0ull;
    return splitmix64(d.seed ^ splitmix64((c << 16) | d.subseq));
}
__device__ __forceinline__ float dropout_factor(const DropoutArgs &d, uint64_t key, int64_t i) {
    return (splitmix64(key + static_cast<uint64_t>(i)) >> 32) >= d.cut ? d.scale : 0.0f;
}

// Host: DropoutArgs of fl_dropout (NULL: off); FL_EINVAL for a bad p or subseq.
int dropout_args(const fl_dropout *drop, DropoutArgs *out);

// ---- workspace carving ---------------------------------------------------
struct Carve {
    char *base;
    size_t size, used;
    __host__ Carve(void *p, size_t n) : base(static_cast<char *>(p)), size(n), used(0) {}
    template <typename T>
    __host__ T *take(size_t count) {
        size_t off = (used + 255) & ~size_t(255);
        used = off + count * sizeof(T);
        return used <= size ? reinterpret_cast<T *>(base + off) : nullptr;
    }
};
template <typename T>
inline size_t carve_bytes(size_t count) { return ((count * sizeof(T) + 255) & ~size_t(255)) + 256; }

// ---- warp / block helpers --------------------------------------------------
__device__ __forceinline__ unsigned lanemask_lt() {
    unsigned m;
    asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
    return m;
}

template <typename T>
__device__ __forceinline__ T warp_sum(T v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
    return v;
}

template <typename T>
__device__ __forceinline__ T warp_max(T v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) { T u = __shfl_xor_sync(kFull, v, o); v = u > v ? u : v; }
    return v;
}

// Inclusive warp scan (fixed order -> deterministic).
template <typename T>
__device__ __forceinline__ T warp_inclusive_scan(T v) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        T u = __shfl_up_sync(kFull, v, o);
        if (lane >= o) v += u;
    }
    return v;
}

// Block-wide exclusive scan of one value per thread; `scratch` holds
// blockDim.x / 32 + 1 elements.  Returns the exclusive prefix; *total gets
// the block total.  All threads must call it.
template <typename T>
__device__ __forceinline__ T block_exclusive_scan(T v, T *scratch, T *total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    T inc = warp_inclusive_scan(v);
    if (lane == 31) scratch[warp] = inc;
    __syncthreads();
    if (warp == 0) {
        T s = lane < nw ? scratch[lane] : T(0);
        T si = warp_inclusive_scan(s);
        if (lane < nw) scratch[lane] = si - s;
        if (lane == nw - 1) scratch[nw] = si;
    }
    __syncthreads();
    T res = scratch[warp] + inc - v;
    *total = scratch[nw];
    __syncthreads();
    return res;
}

// Block-wide sum in a fixed tree (deterministic); result valid in all threads.
template <typename T>
__device__ __forceinline__ T block_sum(T v, T *scratch) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    v = warp_sum(v);
    if (lane == 0) scratch[warp] = v;
    __syncthreads();
    if (warp == 0) {
        T s = lane < nw ? scratch[lane] : T(0);
        s = warp_sum(s);
        if (lane == 0) scratch[nw] = s;
    }
    __syncthreads();
    T r = scratch[nw];
    __syncthreads();
    return r;
}

template <typename T>
__device__ __forceinline__ T block_max(T v, T *scratch) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    v = warp_max(v);
    if (lane == 0) scratch[warp] = v;
    __syncthreads();
    if (warp == 0) {
        T s = lane < nw ? scratch[lane] : T(0);
        s = warp_max(s);
        if (lane == 0) scratch[nw] = s;
    }
    __syncthreads();
    T r = scratch[nw];
    __syncthreads();
    return r;
}

// Order-preserving key of an fp32 value (larger value -> larger key).
__device__ __forceinline__ uint32_t float_order_key(float x) {
    uint32_t u = __float_as_uint(x);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__device__ __forceinline__ uint64_t double_order_key(double x) {
    uint64_t u = static_cast<uint64_t>(__double_as_longlong(x));
    return (u & 0x8000000000000000ull) ? ~u : (u | 0x8000000000000000ull);
}

// ---- exact fixed-point accumulation (order-independent, deterministic) ---
// A value x is accumulated as the 128-bit two's complement integer
// trunc(x * 2^scale); carries between the two 64-bit words are exact, so the
// final sum does not depend on the order of the additions.
struct Fixed128 { unsigned long long lo, hi; };

__device__ __forceinline__ Fixed128 to_fixed(float x, int scale) {
    Fixed128 r{0ull, 0ull};
    uint32_t u = __float_as_uint(x);
    int e = (u >> 23) & 0xff;
    uint32_t mant = u & 0x7fffffu;
    if (e == 0) { if (mant == 0) return r; e = 1; } else mant |= 0x800000u;
    int sh = e - 150 + scale;  // value = mant * 2^(e - 150)
    unsigned long long lo = 0, hi = 0;
    if (sh >= 0) {
        if (sh < 64) {
            lo = static_cast<unsigned long long>(mant) << sh;
            hi = sh == 0 ? 0ull : (sh > 40 ? (static_cast<unsigned long long>(mant) >> (64 - sh)) : 0ull);
        } else if (sh < 128) {
            hi = static_cast<unsigned long long>(mant) << (sh - 64);
        } else {
            hi = 0x7fffffffffffffffull;  // saturate (not reached with a valid scale)
        }
    } else if (sh > -24) {
        lo = static_cast<unsigned long long>(mant >> (-sh));
    }
    if (u & 0x80000000u) {  // negate
        lo = ~lo; hi = ~hi;
        lo += 1ull;
        if (lo == 0ull) hi += 1ull;
    }
    r.lo = lo; r.hi = hi;
    return r;
}

__device__ __forceinline__ void fixed_atomic_add(unsigned long long *acc, Fixed128 v) {
    if (v.lo == 0ull && v.hi == 0ull) return;
    unsigned long long old = atomicAdd(acc, v.lo);
    unsigned long long carry = (old + v.lo < old) ? 1ull : 0ull;
    unsigned long long h = v.hi + carry;
    if (h) atomicAdd(acc + 1, h);
}

// Round a 128-bit fixed-point value to the nearest fp32 (ties to even) and
// scale by 2^-scale.
__device__ __forceinline__ float fixed_to_float(unsigned long long lo, unsigned long long hi, int scale) {
    bool neg = (static_cast<long long>(hi) < 0);
    if (neg) { lo = ~lo; hi = ~hi; lo += 1ull; if (lo == 0ull) hi += 1ull; }
    if (hi == 0ull && lo == 0ull) return 0.0f;
    int lz = hi ? __clzll(static_cast<long long>(hi)) : 64 + __clzll(static_cast<long long>(lo));
    int msb = 127 - lz;                   // index of the leading one
    int drop = msb - 23;                  // bits below the 24-bit mantissa
    float f;
    int exp2;
    if (drop <= 0) {
        f = static_cast<float>(static_cast<uint32_t>(lo));  // exact: < 2^24
        exp2 = -scale;
    } else {
        // 24-bit mantissa of (value >> drop), rounded to nearest, ties to even.
        unsigned long long m, rbit, sticky;
        const int rb = drop - 1;  // rounding bit position
        if (drop >= 64) {
            m = hi >> (drop - 64);
        } else {
            m = (lo >> drop) | (hi << (64 - drop));
        }
        if (rb >= 64) {
            rbit = (hi >> (rb - 64)) & 1ull;
            unsigned long long below_hi = (rb - 64 == 0) ? 0ull : (hi & ((1ull << (rb - 64)) - 1ull));
            sticky = (below_hi | lo) ? 1ull : 0ull;
        } else {
            rbit = (lo >> rb) & 1ull;
            sticky = (rb == 0) ? 0ull : ((lo & ((1ull << rb) - 1ull)) ? 1ull : 0ull);
        }
        m &= 0xffffffull;
        if (rbit && (sticky || (m & 1ull))) m += 1ull;  // may reach 2^24: still exact in fp32
        f = static_cast<float>(static_cast<uint32_t>(m));
        exp2 = drop - scale;
    }
    float r = ldexpf(f, exp2);
    return neg ? -r : r;
}

// Scale such that values with |x| <= bound summed count times stay below
// 2^125.  Returns 0 when bound == 0.
__host__ __device__ inline int fixed_scale_for(float bound, long long count) {
    if (!(bound > 0.0f)) return 0;
    int eb;
    frexpf(bound, &eb);                 // bound < 2^eb
    int ec = 0;
    while ((1ll << ec) <= count && ec < 62) ++ec;  // count < 2^ec
    return 125 - eb - ec;
}

}  // namespace fl
