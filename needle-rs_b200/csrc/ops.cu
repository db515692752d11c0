// The fused row ops of a Needle 3 layer as standalone kernels over [T, d]
// activations: ZC-RMSNorm, RoPE at positions 0..T-1, the MLP's SiLU and the
// CQ embedding gather. In the forward pass these are fused into the mHC
// read, conv, post-block and embedding kernels; here each runs alone so its
// bandwidth can be measured and its arithmetic checked against the
// reference's (crates/needle-engine/src/infer.rs, qlinear.rs). All are HBM
// bound: one read and one write of the rows, 16-byte loads and stores.

#include <cuda_runtime.h>

#include <cmath>
#include <stdexcept>
#include <string>

#include "cqrow.cuh"
#include "kernels.h"
#include "needle_engine.h"
#include "numerics.cuh"

namespace nd {

bool model_embedding(const nd_model* m, DevMat* emb, int* device);
void set_error(const std::string& msg);

static inline int cdiv(int a, int b) { return (a + b - 1) / b; }

// ------------------------------------------------------------------ zcn

// infer.rs:426-443 (zcn) over rows of 768 with infer.rs:372-417 (dot16):
// the sixteen fma chains c (element 16 k + c, k = 0 .. 47 in order) of the
// sum of squares, combined ((A2 + A3) + A1) + A0 per lane then
// (l0 + l1) + (l2 + l3); r = 1 / sqrt(ss / 768 + 1e-6); out = fma(x r, s,
// x r). A warp takes two rows: they arrive as 16-byte loads (kept in
// registers for the output) and through shared memory, where lane c of each
// half-warp runs chain c of its row; rows are padded to 784 floats so the
// two halves read disjoint banks.
constexpr int ZCN_D = 768, ZCN_LD = 784, ZCN_WARPS = 4;

__global__ void __launch_bounds__(32 * ZCN_WARPS) op_zcn_kernel(const float* __restrict__ x, const float* __restrict__ s, int T,
                                                                float* __restrict__ out) {
    __shared__ __align__(16) float rows[ZCN_WARPS][2][ZCN_LD];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int r0 = (blockIdx.x * ZCN_WARPS + warp) * 2;
    if (r0 >= T) return;
    // float4 q = lane + 32 k of the pair: row q / 192, column 4 (q % 192)
    float4 v[12];
#pragma unroll
    for (int k = 0; k < 12; k++) {
        const int q = lane + 32 * k, rr = q / 192, c4 = q % 192;
        v[k] = r0 + rr < T ? __ldg((const float4*)(x + (size_t)(r0 + rr) * ZCN_D) + c4) : make_float4(0.f, 0.f, 0.f, 0.f);
        *(float4*)&rows[warp][rr][4 * c4] = v[k];
    }
    __syncwarp();
    const int hr = lane >> 4, c = lane & 15;
    const float* row = rows[warp][hr];
    float acc = 0.f;
#pragma unroll 16
    for (int k = 0; k < ZCN_D / 16; k++) {
        const float e = row[16 * k + c];
        acc = __fmaf_rn(e, e, acc);
    }
    // chain c = 4 j + l lives on lane 16 hr + c: the combine over the half-warp
    float a[16];
#pragma unroll
    for (int i = 0; i < 16; i++) a[i] = __shfl_sync(0xffffffffu, acc, 16 * hr + i);
    const float r = rinv(dot16_combine(a), ZCN_D);
    const float rA = __shfl_sync(0xffffffffu, r, 0), rB = __shfl_sync(0xffffffffu, r, 16);
#pragma unroll
    for (int k = 0; k < 12; k++) {
        const int q = lane + 32 * k, rr = q / 192, c4 = q % 192;
        if (r0 + rr >= T) continue;
        const float rk = rr ? rB : rA;
        const float4 w = __ldg((const float4*)s + c4);
        float4 o;
        float t;
        t = __fmul_rn(v[k].x, rk); o.x = __fmaf_rn(t, w.x, t);
        t = __fmul_rn(v[k].y, rk); o.y = __fmaf_rn(t, w.y, t);
        t = __fmul_rn(v[k].z, rk); o.z = __fmaf_rn(t, w.z, t);
        t = __fmul_rn(v[k].w, rk); o.w = __fmaf_rn(t, w.w, t);
        *((float4*)(out + (size_t)(r0 + rr) * ZCN_D) + c4) = o;
    }
}

// ----------------------------------------------------------------- RoPE

// The rotation of infer.rs:1474-1483 over a row's 12 q heads and 2 k heads
// (48 wide, halves of 24) with the chunk rows' tables of infer.rs:1716-1744:
// cos, sin = sincosf(freq[f] * pos) (the f32 product, then the f64 sincos
// rounded once: infer.rs:83-102), x[f] = fma(-sin, x[f + 24], cos x[f]),
// x[f + 24] = fma(sin, x[f], cos x[f + 24]). A warp per row: lanes 0-23
// form the row's 24 (cos, sin) pairs, then the 336 rotation pairs are
// spread over the warp.
struct RopeFreq {
    float f[24];
};
constexpr int ROPE_W = 672, ROPE_PAIRS = 14 * 24;

__global__ void __launch_bounds__(256) op_rope_kernel(const float* __restrict__ x, int T, RopeFreq fq, float* __restrict__ out) {
    const int lane = threadIdx.x & 31;
    const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (row >= T) return;
    constexpr int K = (ROPE_PAIRS + 31) / 32;
    const float* xr = x + (size_t)row * ROPE_W;
    float* orow = out + (size_t)row * ROPE_W;
    // the row's values first (independent of the angles), then the sincos
    float a[K], b[K];
#pragma unroll
    for (int k = 0; k < K; k++) {
        const int p = lane + 32 * k, h = p / 24, f = p % 24;
        a[k] = p < ROPE_PAIRS ? __ldg(xr + h * 48 + f) : 0.f;
        b[k] = p < ROPE_PAIRS ? __ldg(xr + h * 48 + f + 24) : 0.f;
    }
    float cs = 0.f, sn = 0.f;
    if (lane < 24) {
        double sd, cd;
        sincos((double)__fmul_rn(fq.f[lane], (float)row), &sd, &cd);
        cs = (float)cd;
        sn = (float)sd;
    }
#pragma unroll
    for (int k = 0; k < K; k++) {
        const int p = lane + 32 * k, h = p / 24, f = p % 24;
        const float c = __shfl_sync(0xffffffffu, cs, f), sv = __shfl_sync(0xffffffffu, sn, f);
        if (p < ROPE_PAIRS) {
            orow[h * 48 + f] = __fmaf_rn(-sv, b[k], __fmul_rn(c, a[k]));
            orow[h * 48 + f + 24] = __fmaf_rn(sv, a[k], __fmul_rn(c, b[k]));
        }
    }
}

// ----------------------------------------------------------------- SiLU

// infer.rs:2463-2496 (silu_native): z / (nexp(-z) + 1), elementwise.
__global__ void __launch_bounds__(256) op_silu_kernel(const float* __restrict__ x, long long n, float* __restrict__ out) {
    const long long n4 = n / 4;
    const long long stride = (long long)gridDim.x * blockDim.x;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += stride) {
        const float4 z = __ldg((const float4*)x + i);
        float4 o;
        o.x = __fdiv_rn(z.x, __fadd_rn(nexp(-z.x), 1.0f));
        o.y = __fdiv_rn(z.y, __fadd_rn(nexp(-z.y), 1.0f));
        o.z = __fdiv_rn(z.z, __fadd_rn(nexp(-z.z), 1.0f));
        o.w = __fdiv_rn(z.w, __fadd_rn(nexp(-z.w), 1.0f));
        ((float4*)out)[i] = o;
    }
    if (blockIdx.x == 0 && threadIdx.x < (n & 3)) {
        const long long i = 4 * n4 + threadIdx.x;
        out[i] = __fdiv_rn(x[i], __fadd_rn(nexp(-x[i]), 1.0f));
    }
}

// --------------------------------------------------------------- gather

// qlinear.rs:309-323 (QMat::row) of the embedding for each id: a warp per
// row. The row's codes and norms for all groups are loaded first (each
// lane's 4 codes of every group), then each group's 128 values are
// dequantized and rotated by the warp and written as one 512-byte run.
constexpr int GATHER_MAXG = 8;

__global__ void __launch_bounds__(256) op_gather_kernel(DevMat emb, const int32_t* __restrict__ ids, int T, float* __restrict__ out) {
    const int lane = threadIdx.x & 31;
    const int t = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (t >= T) return;
    const int id = __ldg(ids + t);
    const bool ok = id >= 0 && id < emb.out;  // an id past the vocabulary gives a row of zeros
    const int d = emb.in_dim, G = emb.groups, width = emb.width, bpg = 16 * width;
    const size_t row = ok ? (size_t)id : 0;
    const uint8_t* codes = emb.codes + row * G * bpg;
    const int bit = 4 * width * lane;
    uint32_t w[GATHER_MAXG];
    float norm[GATHER_MAXG];
#pragma unroll
    for (int g = 0; g < GATHER_MAXG; g++) {
        if (g < G) {
            const uint8_t* c = codes + g * bpg;
            uint32_t v = __ldg(c + (bit >> 3));
            if (width > 2) v |= (uint32_t)__ldg(c + (bit >> 3) + 1) << 8;
            w[g] = v >> (bit & 7);
            norm[g] = h2f(__ldg(emb.norms + row * G + g));
        }
    }
    const uint32_t mask = (1u << width) - 1;
#pragma unroll
    for (int g = 0; g < GATHER_MAXG; g++) {
        if (g >= G) break;
        float v[4];
#pragma unroll
        for (int k = 0; k < 4; k++) v[k] = __fmul_rn(emb.fvals[(w[g] >> (width * k)) & mask], norm[g]);
        fwht128_warp(v, lane);
#pragma unroll
        for (int k = 0; k < 4; k++) v[k] = ok ? __fmul_rn(v[k], ND_HS128) : 0.f;
        const int col = g * 128 + 4 * lane;
        if (col + 3 < d) *(float4*)(out + (size_t)t * d + col) = make_float4(v[0], v[1], v[2], v[3]);
    }
}

static int sm_count_of(int dev) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0) v = 148;
    return v;
}

static void check_launch(const char* what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
    add_launches(1);
}

static void check_aligned(const void* p, const char* what) {
    if (!p) throw std::runtime_error(std::string(what) + ": null pointer");
    if ((uintptr_t)p % 16) throw std::runtime_error(std::string(what) + ": pointers must be 16-byte aligned");
}

}  // namespace nd

using namespace nd;

extern "C" {

int nd_op_zcn(const float* x, const float* s, int T, float* out, void* stream) {
    try {
        check_aligned(x, "nd_op_zcn");
        check_aligned(s, "nd_op_zcn");
        check_aligned(out, "nd_op_zcn");
        if (T < 1) throw std::runtime_error("nd_op_zcn: T must be positive");
        const int rows_per_cta = 2 * ZCN_WARPS;
        op_zcn_kernel<<<cdiv(T, rows_per_cta), 32 * ZCN_WARPS, 0, (cudaStream_t)stream>>>(x, s, T, out);
        check_launch("nd_op_zcn");
        return 0;
    } catch (std::exception& e) {
        set_error(e.what());
        return -1;
    }
}

int nd_op_rope(const float* x, int T, float theta, float* out, void* stream) {
    try {
        if (!x || !out) throw std::runtime_error("nd_op_rope: null pointer");
        if (T < 1) throw std::runtime_error("nd_op_rope: T must be positive");
        if (!(theta > 0.f)) throw std::runtime_error("nd_op_rope: theta must be positive");
        // infer.rs:938-946 (Tables::new): freq[i] = powf(theta, i * (-2 / 48)),
        // the f64 pow rounded once
        RopeFreq fq;
        const float coef = -2.0f / 48.0f;
        for (int i = 0; i < 24; i++) fq.f[i] = (float)std::pow((double)theta, (double)((float)i * coef));
        op_rope_kernel<<<cdiv(T, 8), 256, 0, (cudaStream_t)stream>>>(x, T, fq, out);
        check_launch("nd_op_rope");
        return 0;
    } catch (std::exception& e) {
        set_error(e.what());
        return -1;
    }
}

int nd_op_silu(const float* x, long long n, float* out, void* stream) {
    try {
        check_aligned(x, "nd_op_silu");
        check_aligned(out, "nd_op_silu");
        if (n < 1) throw std::runtime_error("nd_op_silu: n must be positive");
        int dev = 0;
        cudaGetDevice(&dev);
        const long long n4 = std::max(n / 4, 1LL);
        const int grid = (int)std::min<long long>((n4 + 255) / 256, 8LL * sm_count_of(dev));
        op_silu_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(x, n, out);
        check_launch("nd_op_silu");
        return 0;
    } catch (std::exception& e) {
        set_error(e.what());
        return -1;
    }
}

int nd_op_gather(const nd_model* m, const int* ids, int T, float* out, void* stream) {
    try {
        DevMat emb;
        int device = 0;
        if (!m || !ids) throw std::runtime_error("nd_op_gather: null argument");
        check_aligned(out, "nd_op_gather");
        if (!model_embedding(m, &emb, &device)) throw std::runtime_error("nd_op_gather: no model");
        if (emb.in_dim % 128 || emb.groups > GATHER_MAXG)
            throw std::runtime_error("nd_op_gather: d_model must be a multiple of 128, at most 1024");
        if (T < 1) throw std::runtime_error("nd_op_gather: T must be positive");
        int prev = 0;
        cudaGetDevice(&prev);
        cudaSetDevice(device);
        op_gather_kernel<<<cdiv(T, 8), 256, 0, (cudaStream_t)stream>>>(emb, (const int32_t*)ids, T, out);
        cudaError_t e = cudaGetLastError();
        cudaSetDevice(prev);
        if (e != cudaSuccess) throw std::runtime_error(std::string("nd_op_gather: ") + cudaGetErrorString(e));
        add_launches(1);
        return 0;
    } catch (std::exception& e) {
        set_error(e.what());
        return -1;
    }
}

}  // extern "C"
