// Device arithmetic of the Needle 3 packed path, op for op as the reference's
// portable scalar code computes it (crates/needle-engine/src/infer.rs,
// qlinear.rs). Every translation unit is compiled with -fmad=false, so a
// product followed by an add stays two roundings unless written __fmaf_rn,
// and with IEEE division and square root (no fast-math).
#pragma once

#include <cstdint>
#include <cuda_fp16.h>

namespace nd {

// qlinear.rs:40 and infer.rs:30-36
#define ND_K127 __uint_as_float(0x3c010204u)
#define ND_INV_SQRT_QK __uint_as_float(0x3e13cd3au)
#define ND_Q21 __uint_as_float(0x49fffff8u)
#define ND_C21 __uint_as_float(0x35000004u)
#define ND_NEG __uint_as_float(0xf149f2cau)

// infer.rs:83-102: the f32 libm calls are f64 results rounded once.
__device__ __forceinline__ float lexpf(float x) { return (float)exp((double)x); }

// infer.rs:353-366: the engine's inline exp.
__device__ __forceinline__ float nexp(float x) {
    x = fminf(fmaxf(x, __uint_as_float(0xc2b0c0a5u)), __uint_as_float(0x42b0c0a5u));
    float k = rintf(__fmul_rn(x, __uint_as_float(0x3fb8aa3bu)));
    float r = __fmaf_rn(k, __uint_as_float(0xbf318000u), x);
    r = __fmaf_rn(k, __uint_as_float(0x395e8083u), r);
    float p = __fmaf_rn(__uint_as_float(0x39506967u), r, __uint_as_float(0x3ab743ceu));
    p = __fmaf_rn(r, p, __uint_as_float(0x3c088908u));
    p = __fmaf_rn(r, p, __uint_as_float(0x3d2aa9c1u));
    p = __fmaf_rn(r, p, __uint_as_float(0x3e2aaaaau));
    p = __fmaf_rn(r, p, 0.5f);
    float y = __fmaf_rn(__fmul_rn(r, r), p, r);
    float s = __uint_as_float((uint32_t)(((int32_t)k << 23) + 0x3f800000));
    return __fmaf_rn(s, y, s);
}

// infer.rs:421-423
__device__ __forceinline__ float rinv(float ss, int n) {
    return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)n), 1e-6f)));
}

// The combine of infer.rs:372-417 once the sixteen fma chains are known:
// chain c (0..15) is accumulator set j = c / 4, lane l = c % 4.
__device__ __forceinline__ float dot16_combine(const float* a /*[16]*/) {
    float t[4];
#pragma unroll
    for (int l = 0; l < 4; l++) t[l] = __fadd_rn(__fadd_rn(__fadd_rn(a[8 + l], a[12 + l]), a[4 + l]), a[l]);
    return __fadd_rn(__fadd_rn(t[0], t[1]), __fadd_rn(t[2], t[3]));
}

// One of the sixteen chains of dot16 (element i = c*16 + chain, fma from 0)
// over N elements. The operands are loaded BATCH elements at a time before
// their fmas (all of them, by default), so the chain waits on its own fmas,
// not on a shared-memory load per step; kernels short of registers take
// smaller batches.
template <int N, int BATCH = N / 16>
__device__ __forceinline__ float dot16_chain(const float* x, const float* y, int chain) {
    static_assert(N % 16 == 0 && (N / 16) % BATCH == 0, "whole chains and batches");
    float acc = 0.f;
#pragma unroll 1
    for (int e0 = 0; e0 < N / 16; e0 += BATCH) {
        float a[BATCH], b[BATCH];
#pragma unroll
        for (int e = 0; e < BATCH; e++) {
            a[e] = x[chain + 16 * (e0 + e)];
            b[e] = y[chain + 16 * (e0 + e)];
        }
#pragma unroll
        for (int e = 0; e < BATCH; e++) acc = __fmaf_rn(a[e], b[e], acc);
    }
    return acc;
}

// dot16_chain<N>(x, x, chain) with one load per element.
template <int N, int BATCH = N / 16>
__device__ __forceinline__ float dot16_sq(const float* x, int chain) {
    static_assert(N % 16 == 0 && (N / 16) % BATCH == 0, "whole chains and batches");
    float acc = 0.f;
#pragma unroll 1
    for (int e0 = 0; e0 < N / 16; e0 += BATCH) {
        float a[BATCH];
#pragma unroll
        for (int e = 0; e < BATCH; e++) a[e] = x[chain + 16 * (e0 + e)];
#pragma unroll
        for (int e = 0; e < BATCH; e++) acc = __fmaf_rn(a[e], a[e], acc);
    }
    return acc;
}

// The int8 quantizer's rounding: half away from zero, saturated
// (qlinear.rs:113-140).
__device__ __forceinline__ int8_t q8_round(float v, float inv) {
    float r = roundf(__fmul_rn(v, inv));
    if (r != r) return 0;  // NaN: Rust's saturating `as i8` (and NEON's fcvtas) give 0
    r = fminf(fmaxf(r, -128.f), 127.f);
    return (int8_t)(int)r;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

__device__ __forceinline__ int warp_sum_i(int v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// quant.rs:91-115 on one 128-wide group held by a warp, lane i owning
// elements 4i..4i+3: the butterflies of every stage h pair j with j+h, the
// lower keeping a+b and the upper a-b, exactly as the sequential loop does.
__device__ __forceinline__ void fwht128_warp(float v[4], int lane) {
    float a, b;
    a = v[0]; b = v[1]; v[0] = __fadd_rn(a, b); v[1] = __fsub_rn(a, b);
    a = v[2]; b = v[3]; v[2] = __fadd_rn(a, b); v[3] = __fsub_rn(a, b);
    a = v[0]; b = v[2]; v[0] = __fadd_rn(a, b); v[2] = __fsub_rn(a, b);
    a = v[1]; b = v[3]; v[1] = __fadd_rn(a, b); v[3] = __fsub_rn(a, b);
#pragma unroll
    for (int m = 1; m < 32; m <<= 1) {
        bool upper = (lane & m) != 0;
#pragma unroll
        for (int k = 0; k < 4; k++) {
            float o = __shfl_xor_sync(0xffffffffu, v[k], m);
            v[k] = upper ? __fsub_rn(o, v[k]) : __fadd_rn(v[k], o);
        }
    }
}

__device__ __forceinline__ float h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }

}  // namespace nd
