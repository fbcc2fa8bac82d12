// Device helpers shared by the MoE kernels (sm_100a).
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace gtm {

constexpr int kGroup = 64;  // MLX affine quantisation group along the input dimension

__device__ __forceinline__ float bf16f(uint16_t b) { return __uint_as_float(uint32_t(b) << 16); }

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Weights are read once per token and never written by these kernels: non-coherent path,
// no L1 allocation (they are streamed).
__device__ __forceinline__ uint32_t ldg_stream_u32(const void* p) {
    uint32_t v;
    asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(v) : "l"(p));
    return v;
}
__device__ __forceinline__ uint16_t ldg_u16(const void* p) {
    uint16_t v;
    asm volatile("ld.global.nc.u16 %0, [%1];" : "=h"(v) : "l"(p));
    return v;
}
__device__ __forceinline__ uint4 ldg_stream_u4(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
    return v;
}

// ---- exact RMSNorm scale ---------------------------------------------------------------
// The reference forms inv = 1/sqrtf((float)(sum_d / n) + eps) with sum_d a *sequential*
// double sum of x*x (src/cpu_reference.cpp:43-46). A parallel double sum differs from it by
// at most ~(n + depth) ulps of the sum; the float conversion of sum/n agrees with the
// reference's whenever sum/n is farther than that bound from a float rounding midpoint. That
// is checked, and in the rare case it fails the sequential sum is formed by one thread. The
// result is bit-identical with the reference either way. `x` is in shared memory.
// Must be called by all threads of the block; `red` is >= 33 doubles of shared scratch.
__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ inline float exact_rms_inv(const float* x, int n, float eps, double* red) {
    const int tid = threadIdx.x, nth = blockDim.x, lane = tid & 31, warp = tid >> 5;
    const int nwarps = (nth + 31) >> 5;
    double acc = 0.0;
    for (int i = tid; i < n; i += nth) {
        const double v = (double)x[i];
        acc = __dadd_rn(acc, __dmul_rn(v, v));   // v*v is exact in double
    }
    acc = warp_sum_d(acc);
    __syncthreads();                              // `red` may still be read by a previous call
    if (lane == 0) red[warp] = acc;
    __syncthreads();
    if (tid == 0) {
        double s = 0.0;
        for (int w = 0; w < nwarps; ++w) s = __dadd_rn(s, red[w]);
        double q = __ddiv_rn(s, (double)n);
        float f = __double2float_rn(q);
        // rounding midpoints around f
        const double fd = (double)f;
        const double lo = (fd + (double)nextafterf(f, -INFINITY)) * 0.5;
        const double hi = (fd + (double)nextafterf(f, INFINITY)) * 0.5;
        const double bound = q * ((double)n + 48.0) * 1.1102230246251565e-16;  // (n+48) * 2^-53
        if (!(q - lo > bound && hi - q > bound)) {
            // too close to call: reproduce the sequential sum exactly
            double seq = 0.0;
            for (int i = 0; i < n; ++i) {
                const double v = (double)x[i];
                seq = __dadd_rn(seq, __dmul_rn(v, v));
            }
            f = __double2float_rn(__ddiv_rn(seq, (double)n));
        }
        red[32] = (double)__fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(f, eps)));
    }
    __syncthreads();
    return (float)red[32];
}

// ---- bounded grid barrier ----------------------------------------------------------------
// Each CTA publishes the barrier number it reached in its own flag word; every CTA waits until
// all flags reach it. Waits are bounded by `timeout_ns` of %globaltimer; on expiry the error
// word is set and false is returned so the caller unwinds instead of hanging.
struct GridSync {
    unsigned* flags;   // [gridDim.x]
    int* err;          // this launch's error word (0 = ok), cleared before every launch
    int* sticky;       // error word kept until the host reads and clears it
};

__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
// Polling load: relaxed (independent loads stay in flight together); the caller fences once
// after the condition holds.
__device__ __forceinline__ unsigned ld_relaxed(const unsigned* p) {
    unsigned v;
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release(unsigned* p, unsigned v) {
    asm volatile("st.release.gpu.global.u32 [%0], %1;" :: "l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_volatile_int(const int* p) { return *(volatile const int*)p; }

__device__ inline bool grid_barrier(const GridSync& gs, unsigned epoch, uint64_t timeout_ns, int* s_flag) {
    __syncthreads();
    if (threadIdx.x < 32) {
        const int lane = threadIdx.x;
        if (lane == 0) {
            __threadfence();
            st_release(gs.flags + blockIdx.x, epoch);
        }
        __syncwarp();
        const uint64_t t0 = globaltimer_ns();
        bool ok = true;
        for (;;) {
            bool mine = true;
            for (unsigned b = lane; b < gridDim.x; b += 32) mine &= (ld_relaxed(gs.flags + b) >= epoch);
            if (__all_sync(0xffffffffu, mine)) break;
            if (ld_volatile_int(gs.err) != 0) { ok = false; break; }
            if (globaltimer_ns() - t0 > timeout_ns) {
                if (lane == 0) { atomicExch(gs.err, 1); atomicExch(gs.sticky, 1); }
                ok = false;
                break;
            }
            __nanosleep(32);
        }
        __threadfence();
        if (lane == 0) *s_flag = ok ? 0 : 1;
    }
    __syncthreads();
    return *s_flag == 0;
}

// ---- int4 word decode ----------------------------------------------------------------------
// dot = sum_k nibble_k(w) * x_k for one 32-bit word (8 nibbles, low first). Each nibble is
// placed into the mantissa of 1.0f at its natural bit position p (0..16) with one LOP3, the
// 1.0 is removed exactly, and the product with x_k * 2^(23-p) (pre-scaled, exact) is the
// exact nibble * x_k; nibbles 5..7 come from w >> 16. Two accumulators (f32x2 lanes).
struct XSlice {            // one word's activations, pre-scaled per nibble position
    float2 p[4];           // (x0', x4'), (x1', x5'), (x2', x6'), (x3', x7')
};

__device__ __forceinline__ XSlice make_xslice(const float* x8) {
    // nibble k at bit p_k: k<=4 -> p = 4k; k>=5 -> p = 4(k-4) in (w >> 16)
    XSlice s;
    const float sc[8] = {8388608.0f, 524288.0f, 32768.0f, 2048.0f, 128.0f, 524288.0f, 32768.0f, 2048.0f};
    s.p[0] = make_float2(x8[0] * sc[0], x8[4] * sc[4]);
    s.p[1] = make_float2(x8[1] * sc[1], x8[5] * sc[5]);
    s.p[2] = make_float2(x8[2] * sc[2], x8[6] * sc[6]);
    s.p[3] = make_float2(x8[3] * sc[3], x8[7] * sc[7]);
    return s;
}

__device__ __forceinline__ uint32_t lop_or_and(uint32_t a, uint32_t mask, uint32_t orv) {
    uint32_t d;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(mask), "r"(orv));  // (a & b) | c
    return d;
}

__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
    unsigned long long ra, rb, rc, rd;
    ra = *reinterpret_cast<unsigned long long*>(&a);
    rb = *reinterpret_cast<unsigned long long*>(&b);
    rc = *reinterpret_cast<unsigned long long*>(&c);
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(rd) : "l"(ra), "l"(rb), "l"(rc));
    return *reinterpret_cast<float2*>(&rd);
}
__device__ __forceinline__ float2 fadd2(float2 a, float2 b) {
    unsigned long long ra, rb, rd;
    ra = *reinterpret_cast<unsigned long long*>(&a);
    rb = *reinterpret_cast<unsigned long long*>(&b);
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(rd) : "l"(ra), "l"(rb));
    return *reinterpret_cast<float2*>(&rd);
}

__device__ __forceinline__ float dot_word(uint32_t w, const XSlice& xs) {
    const uint32_t one = 0x3F800000u;
    const uint32_t hi = w >> 16;
    const float2 m1 = make_float2(-1.0f, -1.0f);
    float2 a0 = make_float2(__uint_as_float(lop_or_and(w, 0x0000000Fu, one)), __uint_as_float(lop_or_and(w, 0x000F0000u, one)));
    float2 a1 = make_float2(__uint_as_float(lop_or_and(w, 0x000000F0u, one)), __uint_as_float(lop_or_and(hi, 0x000000F0u, one)));
    float2 a2 = make_float2(__uint_as_float(lop_or_and(w, 0x00000F00u, one)), __uint_as_float(lop_or_and(hi, 0x00000F00u, one)));
    float2 a3 = make_float2(__uint_as_float(lop_or_and(w, 0x0000F000u, one)), __uint_as_float(lop_or_and(hi, 0x0000F000u, one)));
    a0 = fadd2(a0, m1); a1 = fadd2(a1, m1); a2 = fadd2(a2, m1); a3 = fadd2(a3, m1);
    float2 acc = make_float2(0.0f, 0.0f);
    acc = ffma2(a0, xs.p[0], acc);
    acc = ffma2(a1, xs.p[1], acc);
    acc = ffma2(a2, xs.p[2], acc);
    acc = ffma2(a3, xs.p[3], acc);
    return acc.x + acc.y;
}

// Sum of 32 per-lane values v[r] across the warp, one result per lane: after the call lane
// r holds sum over lanes of v[r] (r = 0..31). 31 shuffles per lane.
template <int R>
__device__ __forceinline__ float warp_transpose_reduce(float (&v)[R]) {
    static_assert(R == 32, "transpose reduce expects 32 values");
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int half = 16; half >= 1; half >>= 1) {
        const bool upper = (lane & half) != 0;
#pragma unroll
        for (int i = 0; i < half; ++i) {
            // keep v[i] (lower) or v[i+half] (upper); send the other
            const float send = upper ? v[i] : v[i + half];
            const float keep = upper ? v[i + half] : v[i];
            v[i] = keep + __shfl_xor_sync(0xffffffffu, send, half);
        }
    }
    return v[0];
}

}  // namespace gtm
