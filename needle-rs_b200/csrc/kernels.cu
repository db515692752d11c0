// Kernels of the Needle 3 packed forward pass (sm_100a).
//
// Each kernel reproduces one phase of the reference's native path
// (crates/needle-engine/src/infer.rs `chunk_native`/`layer_native`) for every
// row of a step at once. Integer sums are exact, so their order is free; every
// float op follows the reference's order, rounding and fusion.

#include <atomic>

#include "kernels.h"
#include "numerics.cuh"

namespace nd {

static std::atomic<long long> g_launches{0};
long long launch_count() { return g_launches.load(); }
#define COUNT_LAUNCH() g_launches.fetch_add(1, std::memory_order_relaxed)

__constant__ int8_t c_vals[16];   // code -> int8 codebook value (qlinear.rs:244-265)
__constant__ float c_fvals[16];   // code -> f32 codebook value
__constant__ float c_cbs;         // int8 codebook scale
__constant__ float c_hs128;       // (float)(1/sqrt(128)), quant.rs:71-73

__global__ void cq_gemm_kernel(DevMat W, const int8_t* act, const float* sx, int M, int T, float* y, int ldy, int col0);
static cudaError_t init_attrs();

void set_constants(const int8_t vals[16], const float fvals[16], float cbs, float hs128) {
    init_attrs();
    cudaMemcpyToSymbol(c_vals, vals, 16);
    cudaMemcpyToSymbol(c_fvals, fvals, 64);
    cudaMemcpyToSymbol(c_cbs, &cbs, 4);
    cudaMemcpyToSymbol(c_hs128, &hs128, 4);
}

static inline int cdiv(int a, int b) { return (a + b - 1) / b; }

// --------------------------------------------------------------- tokens

__global__ void write_tokens_kernel(const int32_t* ids, int S, int T, int p0, int32_t* tokens, int cap) {
    int m = blockIdx.x * blockDim.x + threadIdx.x;
    if (m >= S * T) return;
    int s = m / T, i = m % T;
    tokens[(size_t)s * cap + p0 + i] = ids[m];
}

void launch_write_tokens(const int32_t* ids, int S, int T, int p0, Caches c, cudaStream_t st) {
    COUNT_LAUNCH();
    write_tokens_kernel<<<cdiv(S * T, 256), 256, 0, st>>>(ids, S, T, p0, c.tokens, c.cap);
}

// ------------------------------------------------------- CQ row dequant

// QMat::row (qlinear.rs:309-323) of one 128-wide group, by a warp: each
// lane's four weights `fvals[code] * norm`, then the rotation.
__device__ __forceinline__ void cq_group_row(const uint8_t* codes, const uint16_t* norms, size_t row, int groups, int g,
                                             int lane, float v[4]) {
    const uint8_t* c = codes + (row * groups + g) * 64 + 2 * lane;
    uint32_t w = (uint32_t)c[0] | ((uint32_t)c[1] << 8);
    float norm = h2f(norms[row * groups + g]);
#pragma unroll
    for (int k = 0; k < 4; k++) v[k] = __fmul_rn(c_fvals[(w >> (4 * k)) & 15], norm);
    fwht128_warp(v, lane);
#pragma unroll
    for (int k = 0; k < 4; k++) v[k] = __fmul_rn(v[k], c_hs128);
}

// infer.rs:1185-1194: the embedding row times sqrt(d), in every lane.
__global__ void embed_kernel(DevMat emb, const int32_t* ids, float* xs, float scale) {
    int m = blockIdx.x, g = blockIdx.y, lane = threadIdx.x;
    int tok = ids[m];
    float v[4];
    cq_group_row(emb.codes, emb.norms, (size_t)tok, emb.groups, g, lane, v);
    float4 o = make_float4(__fmul_rn(v[0], scale), __fmul_rn(v[1], scale), __fmul_rn(v[2], scale), __fmul_rn(v[3], scale));
    const int d = emb.in_dim;
#pragma unroll
    for (int ln = 0; ln < 4; ln++) *(float4*)(xs + (size_t)m * 4 * d + ln * d + g * 128 + 4 * lane) = o;
}

void launch_embed(DevMat emb, const int32_t* ids, int M, float* xs, cudaStream_t st) {
    COUNT_LAUNCH();
    float scale = __builtin_sqrtf((float)emb.in_dim);
    embed_kernel<<<dim3(M, emb.groups), 32, 0, st>>>(emb, ids, xs, scale);
}

// ------------------------------------------------------------ A8 prep

// prep_group (qlinear.rs:152-164): zero-pad, rotate, int8 with one scale per
// (row, group). Stored in natural order.
__device__ __forceinline__ void prep_group_warp(float v[4], int lane, int8_t* q, float* sx) {
    fwht128_warp(v, lane);
    float a = 0.f;
#pragma unroll
    for (int k = 0; k < 4; k++) {
        v[k] = __fmul_rn(v[k], c_hs128);
        a = fmaxf(a, fabsf(v[k]));
    }
    a = warp_max(a);
    float s = a > 0.f ? __fmul_rn(a, ND_K127) : 1.0f;
    float inv = __fdiv_rn(1.0f, s);
    char4 o;
    o.x = q8_round(v[0], inv);
    o.y = q8_round(v[1], inv);
    o.z = q8_round(v[2], inv);
    o.w = q8_round(v[3], inv);
    *(char4*)(q + 4 * lane) = o;
    if (lane == 0) *sx = s;
}

__global__ void prep_act_kernel(const float* x, int ldx, int K, int8_t* act, float* sx, int G) {
    int m = blockIdx.x, g = blockIdx.y, lane = threadIdx.x;
    float v[4];
#pragma unroll
    for (int k = 0; k < 4; k++) {
        int col = g * 128 + 4 * lane + k;
        v[k] = col < K ? x[(size_t)m * ldx + col] : 0.f;
    }
    prep_group_warp(v, lane, act + ((size_t)m * G + g) * 128, sx + (size_t)m * G + g);
}

void launch_prep_act(const float* x, int ldx, int K, int M, int8_t* act, float* sx, cudaStream_t st) {
    COUNT_LAUNCH();
    int G = cdiv(K, 128);
    prep_act_kernel<<<dim3(M, G), 32, 0, st>>>(x, ldx, K, act, sx, G);
}

// ----------------------------------------------------------- CQ matmul

// The decode combine (qlinear.rs:340-350) for T == 1: four float lanes per
// output, lane l fed by inputs p with (p % 32) / 8 == l, scale
// (sx * cbs) * norm, lanes summed (l0 + l1) + (l2 + l3). The prefill
// combine (qlinear.rs:353-363) otherwise: one fma chain over groups, scale
// (norm * cbs) * sx for a sequence's first T/4*4 rows, norm * (cbs * sx)
// for the rest.
constexpr int GEMM_TN = 64, GEMM_TM = 16, GEMM_K = 768, GEMM_LD = GEMM_K + 4;

__global__ void __launch_bounds__(256) cq_gemm_kernel(DevMat W, const int8_t* act, const float* sx, int M, int T, float* y,
                                                      int ldy, int col0) {
    extern __shared__ __align__(16) int8_t smem[];
    int8_t* ws = smem;                               // [TN][LD]
    int8_t* as = smem + GEMM_TN * GEMM_LD;           // [TM][LD]
    float* sxs = (float*)(as + GEMM_TM * GEMM_LD);   // [TM][6]
    float* nrm = sxs + GEMM_TM * 6;                  // [TN][6]
    const int G = W.groups;
    const int n0 = blockIdx.x * GEMM_TN, m0 = blockIdx.y * GEMM_TM;
    const int tid = threadIdx.x;
    // weights: codes through the LUT into int8, natural order
    for (int idx = tid; idx < GEMM_TN * G * 16; idx += 256) {
        int r = idx / (G * 16), wdx = idx % (G * 16);
        int n = n0 + r;
        uint32_t c = 0;
        if (n < W.out) c = *(const uint32_t*)(W.codes + (size_t)n * G * 64 + wdx * 4);
        char4 lo, hi;
        lo.x = c_vals[c & 15]; lo.y = c_vals[(c >> 4) & 15]; lo.z = c_vals[(c >> 8) & 15]; lo.w = c_vals[(c >> 12) & 15];
        hi.x = c_vals[(c >> 16) & 15]; hi.y = c_vals[(c >> 20) & 15]; hi.z = c_vals[(c >> 24) & 15]; hi.w = c_vals[c >> 28];
        *(char4*)(ws + r * GEMM_LD + wdx * 8) = lo;
        *(char4*)(ws + r * GEMM_LD + wdx * 8 + 4) = hi;
    }
    for (int idx = tid; idx < GEMM_TN * G; idx += 256) {
        int r = idx / G, g = idx % G, n = n0 + r;
        nrm[r * 6 + g] = n < W.out ? h2f(W.norms[(size_t)n * G + g]) : 0.f;
    }
    for (int idx = tid; idx < GEMM_TM * G * 32; idx += 256) {
        int r = idx / (G * 32), wdx = idx % (G * 32);
        int m = m0 + r;
        uint32_t a = m < M ? *(const uint32_t*)(act + (size_t)m * G * 128 + wdx * 4) : 0u;
        *(uint32_t*)(as + r * GEMM_LD + wdx * 4) = a;
    }
    for (int idx = tid; idx < GEMM_TM * G; idx += 256) {
        int r = idx / G, g = idx % G, m = m0 + r;
        sxs[r * 6 + g] = m < M ? sx[(size_t)m * G + g] : 0.f;
    }
    __syncthreads();
    const int nl = tid % GEMM_TN, mq = tid / GEMM_TN;  // 4 rows of m each
    const float cbs = c_cbs;
    float lanes[4][4];
    float acc[4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        acc[i] = 0.f;
#pragma unroll
        for (int l = 0; l < 4; l++) lanes[i][l] = 0.f;
    }
    const int8_t* wr = ws + nl * GEMM_LD;
    for (int g = 0; g < G; g++) {
        int32_t s[4][4];
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
            for (int l = 0; l < 4; l++) s[i][l] = 0;
#pragma unroll
        for (int blk = 0; blk < 4; blk++)
#pragma unroll
            for (int l = 0; l < 4; l++) {
                int off = g * 128 + blk * 32 + l * 8;
                int w0 = *(const int*)(wr + off), w1 = *(const int*)(wr + off + 4);
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    const int8_t* ar = as + (mq * 4 + i) * GEMM_LD + off;
                    s[i][l] = __dp4a(w0, *(const int*)ar, s[i][l]);
                    s[i][l] = __dp4a(w1, *(const int*)(ar + 4), s[i][l]);
                }
            }
        float norm = nrm[nl * 6 + g];
#pragma unroll
        for (int i = 0; i < 4; i++) {
            int ml = mq * 4 + i;
            float sxv = sxs[ml * 6 + g];
            if (T == 1) {
                float sc = __fmul_rn(__fmul_rn(sxv, cbs), norm);
#pragma unroll
                for (int l = 0; l < 4; l++) lanes[i][l] = __fmaf_rn((float)s[i][l], sc, lanes[i][l]);
            } else {
                int ti = (m0 + ml) % T;
                bool block = ti < T / 4 * 4;
                float sc = block ? __fmul_rn(__fmul_rn(norm, cbs), sxv) : __fmul_rn(norm, __fmul_rn(cbs, sxv));
                int tot = s[i][0] + s[i][1] + s[i][2] + s[i][3];
                acc[i] = __fmaf_rn((float)tot, sc, acc[i]);
            }
        }
    }
    int n = n0 + nl;
    if (n >= W.out) return;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        int m = m0 + mq * 4 + i;
        if (m >= M) continue;
        float v = T == 1 ? __fadd_rn(__fadd_rn(lanes[i][0], lanes[i][1]), __fadd_rn(lanes[i][2], lanes[i][3])) : acc[i];
        y[(size_t)m * ldy + col0 + n] = v;
    }
}

static const size_t GEMM_SMEM = (GEMM_TN + GEMM_TM) * GEMM_LD + (GEMM_TM + GEMM_TN) * 6 * 4;

void launch_cq_gemm(DevMat W, const int8_t* act, const float* sx, int M, int T, float* y, int ldy, int col0, cudaStream_t st) {
    COUNT_LAUNCH();
    cq_gemm_kernel<<<dim3(cdiv(W.out, GEMM_TN), cdiv(M, GEMM_TM)), 256, GEMM_SMEM, st>>>(W, act, sx, M, T, y, ldy, col0);
}

static cudaError_t init_attrs() {
    return cudaFuncSetAttribute(cq_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)GEMM_SMEM);
}

// ---------------------------------------------------------------- engram

// infer.rs:1257-1277: the n-gram hash of each (order, head) picks a table
// row; rows the position is too young for stay zero.
__global__ void engram_gather_kernel(DevMat tables, const int32_t* tokens, int cap, int T, int p0, int slots, float* e) {
    int m = blockIdx.x, tbl = blockIdx.y, lane = threadIdx.x;
    const int heads = 3, stride = 3, sub = 128, d = 768;
    int s = m / T, i = m % T, pos = p0 + i;
    int oi = tbl / heads, h = tbl % heads, order = oi == 0 ? 2 : 3;
    float v[4] = {0.f, 0.f, 0.f, 0.f};
    if (pos + 1 >= order) {
        uint32_t acc = 0x9E3779B9u * (uint32_t)(oi * stride + h + 1);
        for (int j = 0; j < order; j++) {
            uint32_t tok = pos >= j ? (uint32_t)tokens[(size_t)s * cap + pos - j] : 0u;
            acc = (acc ^ tok) * 0x01000193u;
        }
        acc ^= acc >> 15;
        size_t row = (size_t)tbl * slots + acc % (uint32_t)slots;
        cq_group_row(tables.codes, tables.norms, row, tables.groups, 0, lane, v);
    }
    *(float4*)(e + (size_t)m * d + tbl * sub + 4 * lane) = make_float4(v[0], v[1], v[2], v[3]);
}

void launch_engram_gather(DevMat tables, Caches c, int S, int T, int p0, int slots, float* e, cudaStream_t st) {
    COUNT_LAUNCH();
    engram_gather_kernel<<<dim3(S * T, 6), 32, 0, st>>>(tables, c.tokens, c.cap, T, p0, slots, e);
}

// infer.rs:1283-1303: the value half of kv, int8 in 32-wide groups, into
// the site's history at the row's position.
__global__ void engram_vhist_kernel(const float* kv, int8_t* ev8, float* evs, int site, int nsites, int T, int p0) {
    int m = blockIdx.x, g = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int s = m / T, pos = p0 + m % T;
    float v = kv[(size_t)m * 1536 + 768 + g * 32 + lane];
    float a = warp_max(fabsf(v));
    float sc = a > 0.f ? __fmul_rn(a, ND_K127) : 1.0f;
    float inv = __fdiv_rn(1.0f, sc);
    size_t slot = ((size_t)s * nsites + site) * ENG_RING + pos % ENG_RING;
    ev8[slot * 768 + g * 32 + lane] = q8_round(v, inv);
    if (lane == 0) evs[slot * 24 + g] = sc;
}

void launch_engram_vhist(const float* kv, Caches c, int site, int nsites, int S, int T, int p0, cudaStream_t st) {
    COUNT_LAUNCH();
    engram_vhist_kernel<<<S * T, 768, 0, st>>>(kv, c.ev8, c.evs, site, nsites, T, p0);
}

// infer.rs:1310-1323 with engram_tap (663-687): four taps at dilation 3,
// each an fma from the int8 history.
__global__ void engram_conv_kernel(const float* taps, const int8_t* ev8, const float* evs, int site, int nsites, int T, int p0,
                                   float* v) {
    int m = blockIdx.x, ch = threadIdx.x;
    int s = m / T, pos = p0 + m % T;
    float o = 0.f;
    for (int j = 0; j < 4; j++) {
        int p = pos - 3 * j;
        if (p < 0) break;
        size_t slot = ((size_t)s * nsites + site) * ENG_RING + p % ENG_RING;
        float deq = __fmul_rn(evs[slot * 24 + ch / 32], (float)ev8[slot * 768 + ch]);
        o = __fmaf_rn(taps[j * 768 + ch], deq, o);
    }
    v[(size_t)m * 768 + ch] = o;
}

void launch_engram_conv(const float* taps, Caches c, int site, int nsites, int S, int T, int p0, float* v, cudaStream_t st) {
    COUNT_LAUNCH();
    engram_conv_kernel<<<S * T, 768, 0, st>>>(taps, c.ev8, c.evs, site, nsites, T, p0, v);
}

// ------------------------------------------------------------ mHC read

// infer.rs:1359-1393: lanes normalized by one rms, int8 (no rotation), the
// 24 int8 gate dots, the pre gates, and the mixed block input u.
__global__ void __launch_bounds__(256) mhc_read_kernel(LayerW w, int lane_own, const float* xs, float* u, float* p) {
    __shared__ __align__(16) float x[3072];
    __shared__ __align__(16) float nx[3072];
    __shared__ __align__(16) int8_t q8[3072];
    __shared__ float part[16];
    __shared__ float red[8];
    __shared__ float pr[24];
    __shared__ float hp[4];
    __shared__ float sc_s[2];
    const int m = blockIdx.x, tid = threadIdx.x;
    const float* xr = xs + (size_t)m * 3072;
    for (int k = tid; k < 768; k += 256) *(float4*)(x + 4 * k) = *(const float4*)(xr + 4 * k);
    __syncthreads();
    if (tid < 16) part[tid] = dot16_chain(x, x, 3072, tid);
    __syncthreads();
    if (tid == 0) sc_s[0] = rinv(dot16_combine(part), 3072);
    __syncthreads();
    float r = sc_s[0], a = 0.f;
    for (int k = tid; k < 3072; k += 256) {
        float v = __fmul_rn(x[k], r);
        nx[k] = v;
        a = fmaxf(a, fabsf(v));
    }
    a = warp_max(a);
    if ((tid & 31) == 0) red[tid >> 5] = a;
    __syncthreads();
    if (tid == 0) {
        float mx = 0.f;
        for (int k = 0; k < 8; k++) mx = fmaxf(mx, red[k]);
        sc_s[1] = mx > 0.f ? __fmul_rn(mx, ND_K127) : 1.0f;
    }
    __syncthreads();
    float sxv = sc_s[1], inv = __fdiv_rn(1.0f, sxv);
    for (int k = tid; k < 3072; k += 256) q8[k] = q8_round(nx[k], inv);
    __syncthreads();
    const int warp = tid >> 5, ln = tid & 31;
    for (int k = warp; k < 24; k += 8) {
        const int* wq = (const int*)(w.phi_q + (size_t)k * 3072);
        int acc = 0;
        for (int j = ln; j < 768; j += 32) acc = __dp4a(wq[j], ((const int*)q8)[j], acc);
        acc = warp_sum_i(acc);
        if (ln == 0) pr[k] = __fmul_rn(__fmul_rn(sxv, w.phi_s[k]), (float)acc);
    }
    __syncthreads();
    if (tid < 4) {
        float off = tid == lane_own ? 4.0f : -4.0f;
        float z = __fadd_rn(__fadd_rn(__fmul_rn(pr[tid], w.a_pre), off), w.b_pre[tid]);
        hp[tid] = __fdiv_rn(1.0f, __fadd_rn(lexpf(-z), 1.0f));
    }
    if (tid < 24) p[(size_t)m * 24 + tid] = pr[tid];
    __syncthreads();
    for (int ch = tid; ch < 768; ch += 256) {
        float o = __fmul_rn(x[ch], hp[0]);
        o = __fmaf_rn(x[768 + ch], hp[1], o);
        o = __fmaf_rn(x[1536 + ch], hp[2], o);
        o = __fmaf_rn(x[2304 + ch], hp[3], o);
        u[(size_t)m * 768 + ch] = o;
    }
}

void launch_mhc_read(LayerW w, int lane, const float* xs, int M, float* u, float* p, cudaStream_t st) {
    COUNT_LAUNCH();
    mhc_read_kernel<<<M, 256, 0, st>>>(w, lane, xs, u, p);
}

// ------------------------------------------------ engram gate + input norm

// infer.rs:1397-1426: the engram gate (when the layer has a site), the
// input ZC-RMSNorm, and A8 of the normed row.
__global__ void __launch_bounds__(256) input_norm_kernel(LayerW w, const float* u, const float* ekv, const float* evals,
                                                         float* x1o, int8_t* act, float* sx) {
    __shared__ __align__(16) float x1[768];
    __shared__ __align__(16) float a[768];
    __shared__ __align__(16) float b[768];
    __shared__ float part[32];
    __shared__ float sc[4];
    const int m = blockIdx.x, tid = threadIdx.x;
    for (int k = tid; k < 768; k += 256) x1[k] = u[(size_t)m * 768 + k];
    __syncthreads();
    if (ekv) {
        const float* kr = ekv + (size_t)m * 1536;
        for (int k = tid; k < 768; k += 256) b[k] = kr[k];
        __syncthreads();
        if (tid < 16) part[tid] = dot16_chain(x1, x1, 768, tid);
        else if (tid < 32) part[tid] = dot16_chain(b, b, 768, tid - 16);
        __syncthreads();
        if (tid == 0) {
            sc[0] = rinv(dot16_combine(part), 768);
            sc[1] = rinv(dot16_combine(part + 16), 768);
        }
        __syncthreads();
        for (int k = tid; k < 768; k += 256) {
            a[k] = __fmul_rn(x1[k], sc[0]);
            b[k] = __fmul_rn(b[k], sc[1]);
        }
        __syncthreads();
        if (tid < 16) part[tid] = dot16_chain(a, b, 768, tid);
        __syncthreads();
        if (tid == 0) {
            float dab = dot16_combine(part);
            sc[2] = __fdiv_rn(1.0f, __fadd_rn(lexpf(__fdiv_rn(-dab, __fsqrt_rn(768.0f))), 1.0f));
        }
        __syncthreads();
        float alpha = sc[2];
        for (int k = tid; k < 768; k += 256) x1[k] = __fmaf_rn(evals[(size_t)m * 768 + k], alpha, x1[k]);
        __syncthreads();
    }
    if (tid < 16) part[tid] = dot16_chain(x1, x1, 768, tid);
    __syncthreads();
    if (tid == 0) sc[3] = rinv(dot16_combine(part), 768);
    __syncthreads();
    float r = sc[3];
    for (int k = tid; k < 768; k += 256) {
        x1o[(size_t)m * 768 + k] = x1[k];
        float t = __fmul_rn(x1[k], r);
        a[k] = __fmaf_rn(t, w.norm_in[k], t);
    }
    __syncthreads();
    const int warp = tid >> 5, ln = tid & 31;
    if (warp < 6) {
        float v[4];
#pragma unroll
        for (int k = 0; k < 4; k++) v[k] = a[warp * 128 + 4 * ln + k];
        prep_group_warp(v, ln, act + ((size_t)m * 6 + warp) * 128, sx + (size_t)m * 6 + warp);
    }
}

void launch_input_norm(LayerW w, const float* u, const float* ekv, const float* evals, int M, float* x1, int8_t* act,
                       float* sx, cudaStream_t st) {
    COUNT_LAUNCH();
    input_norm_kernel<<<M, 256, 0, st>>>(w, u, ekv, evals, x1, act, sx);
}

// ------------------------------------------------ conv taps, RoPE, int8 KV

// infer.rs:1430-1526 (chunk rows) as unit work (infer/step.rs:468-516): per
// row, 12 q heads, 2 k heads and 2 v heads, one warp each. The taps read
// earlier rows of this chunk, else the pre-tap history, else zeros.
__global__ void __launch_bounds__(512) conv_rope_kv_kernel(LayerW w, int l, const float* proj, Caches c, int T, int p0,
                                                           int hist_base, const float* cosr, const float* sinr, float* qbuf) {
    __shared__ float buf[16][64];
    const int m = blockIdx.x, unit = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int s = m / T, i = m % T, pos = p0 + i;
    int start, cw, cc, len;
    const float* wt;
    if (unit < 12) { start = unit * 48; cw = 576; cc = unit * 48; len = 48; wt = w.q_taps; }
    else if (unit < 14) { int kh = unit - 12; start = 576 + kh * 48; cw = 96; cc = kh * 48; len = 48; wt = w.k_taps; }
    else { int vh = unit - 14; start = 672 + vh * 64; cw = 128; cc = vh * 64; len = 64; wt = w.v_taps; }
    const size_t hrow0 = ((size_t)s * c.L + l) * HIST_RING;
    float* x = buf[unit];
    for (int k = lane; k < len; k += 32) {
        float cur = proj[(size_t)m * 1568 + start + k];
        float o = __fmul_rn(wt[cc + k], cur);
        for (int j = 1; j < 3; j++) {
            float wj = wt[j * cw + cc + k];
            int pj = pos - j;
            if (i - j >= 0) {
                o = __fmaf_rn(wj, proj[(size_t)(m - j) * 1568 + start + k], o);
            } else if (pj >= hist_base && pj >= 0) {
                o = __fmaf_rn(wj, c.hist[(hrow0 + pj % HIST_RING) * 800 + start + k], o);
            } else {
                o = __fmaf_rn(wj, 0.0f, o);
            }
        }
        x[k] = o;
    }
    __syncwarp();
    if (unit < 14) {
        // zcn_inplace (infer.rs:446-452) over the 48-wide head, dot16 order.
        float part = 0.f;
        if (lane < 16) {
            part = __fmaf_rn(x[lane], x[lane], 0.f);
            part = __fmaf_rn(x[lane + 16], x[lane + 16], part);
            part = __fmaf_rn(x[lane + 32], x[lane + 32], part);
        }
        float chains[16];
#pragma unroll
        for (int k = 0; k < 16; k++) chains[k] = __shfl_sync(0xffffffffu, part, k);
        float r = rinv(dot16_combine(chains), 48);
        const float* scale = unit < 12 ? w.q_norm : w.k_norm;
        float t0 = __fmul_rn(x[lane], r);
        float y0 = __fmaf_rn(t0, scale[lane], t0);
        float y1 = 0.f;
        if (lane < 16) {
            float t1 = __fmul_rn(x[lane + 32], r);
            y1 = __fmaf_rn(t1, scale[lane + 32], t1);
        }
        __syncwarp();
        x[lane] = y0;
        if (lane < 16) x[lane + 32] = y1;
        __syncwarp();
        // RoPE (infer.rs:1479-1483) on halves of 24.
        float na = 0.f, nb = 0.f;
        if (lane < 24) {
            float cs = cosr[i * 24 + lane], sn = sinr[i * 24 + lane];
            float av = x[lane], bv = x[lane + 24];
            na = __fmaf_rn(-sn, bv, __fmul_rn(cs, av));
            nb = __fmaf_rn(sn, av, __fmul_rn(cs, bv));
        }
        __syncwarp();
        if (lane < 24) {
            x[lane] = na;
            x[lane + 24] = nb;
        }
        __syncwarp();
    }
    if (unit < 12) {
        for (int k = lane; k < 48; k += 32) qbuf[(size_t)m * 576 + unit * 48 + k] = x[k];
        return;
    }
    // int8 KV at this position's slot (infer.rs:1508-1525).
    float a = 0.f;
    for (int k = lane; k < len; k += 32) a = fmaxf(a, fabsf(x[k]));
    a = warp_max(a);
    float sc = a > 0.f ? __fmul_rn(a, ND_K127) : 1.0f;
    float inv = __fdiv_rn(1.0f, sc);
    if (unit < 14) {
        int kh = unit - 12;
        size_t row = (((size_t)s * c.L + l) * 2 + kh) * c.cap + pos;
        for (int k = lane; k < 48; k += 32) c.k8[row * 48 + k] = q8_round(x[k], inv);
        if (lane == 0) c.ks[row] = sc;
    } else {
        int vh = unit - 14;
        size_t row = (((size_t)s * c.L + l) * 2 + vh) * c.cap + pos;
        for (int k = lane; k < 64; k += 32) c.v8[row * 64 + k] = q8_round(x[k], inv);
        if (lane == 0) c.vs[row] = sc;
    }
}

void launch_conv_rope_kv(LayerW w, int l, const float* proj, Caches c, int S, int T, int p0, int hist_base, const float* cosr,
                         const float* sinr, float* qbuf, cudaStream_t st) {
    COUNT_LAUNCH();
    conv_rope_kv_kernel<<<S * T, 512, 0, st>>>(w, l, proj, c, T, p0, hist_base, cosr, sinr, qbuf);
}

// The pre-tap rows of this step into the history ring (after every row has
// read its taps).
__global__ void hist_update_kernel(const float* proj, Caches c, int l, int T, int p0) {
    int s = blockIdx.x, i = T - 1 - blockIdx.y;
    if (i < 0) return;
    int pos = p0 + i;
    size_t dst = (((size_t)s * c.L + l) * HIST_RING + pos % HIST_RING) * 800;
    const float* src = proj + ((size_t)s * T + i) * 1568;
    for (int k = threadIdx.x; k < 800; k += blockDim.x) c.hist[dst + k] = src[k];
}

void launch_hist_update(const float* proj, Caches c, int l, int S, int T, int p0, cudaStream_t st) {
    COUNT_LAUNCH();
    hist_update_kernel<<<dim3(S, T < HIST_RING ? T : HIST_RING), 256, 0, st>>>(proj, c, l, T, p0);
}

// ------------------------------------------------------------- attention

// attend_head_ref (infer.rs:1871-2004) for one (row, head): int8 query,
// the engine's key chunks (key_chunks, 2093-2101), scores with the 4-block
// order rule, chunk_exp (2222-2318), 21-bit digits (2171-2217), integer P.V,
// and the merge (2143-2166); then the gate (1548-1552).
constexpr int ATT_MAXCHUNK = 256, ATT_MAXPARTS = 16;

__device__ __forceinline__ void key_chunks_dev(int n, bool nested, int* count, int* chunk) {
    int k = nested ? 1 : 4;  // (2 * NATIVE_TEAM / nkv).max(1), NATIVE_TEAM = 4, nkv = 2
    int c = (n + 255) / 256;
    if (k * 64 <= n && c < k) c = k;
    int cm = c > 1 ? c : 1;
    int ch = ((n + cm - 1) / cm + 15) / 16 * 16;
    *chunk = ch;
    *count = ch > 0 ? (n + ch - 1) / ch : 0;
}

__global__ void __launch_bounds__(128) attention_kernel(const float* qbuf, const float* proj, Caches c, int l, int T, int p0,
                                                        int window, float* att) {
    __shared__ __align__(16) int8_t q8[48];
    __shared__ float sbuf[ATT_MAXCHUNK];
    __shared__ int8_t dh[ATT_MAXCHUNK], dm_[ATT_MAXCHUNK], dl[ATT_MAXCHUNK];
    __shared__ float red[4];
    __shared__ float pm[ATT_MAXPARTS], psum[ATT_MAXPARTS];
    __shared__ float po[ATT_MAXPARTS][64];
    __shared__ int pv[3][2][64];
    __shared__ float qs_s, m_s, sum_s, wmax_s;
    const int m = blockIdx.x, hh = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int s = m / T, i = m % T, pos = p0 + i, kvh = hh / 6;
    const bool nested = T > 1;
    const int lo = window > 0 ? max(0, pos + 1 - window) : 0;
    const int n = pos + 1 - lo;
    if (warp == 0) {
        float x0 = qbuf[(size_t)m * 576 + hh * 48 + lane];
        float x1 = lane < 16 ? qbuf[(size_t)m * 576 + hh * 48 + 32 + lane] : 0.f;
        float a = warp_max(fmaxf(fabsf(x0), fabsf(x1)));
        float sc = a > 0.f ? __fmul_rn(a, ND_K127) : 1.0f;
        float inv = __fdiv_rn(1.0f, sc);
        q8[lane] = q8_round(x0, inv);
        if (lane < 16) q8[32 + lane] = q8_round(x1, inv);
        if (lane == 0) qs_s = __fmul_rn(sc, ND_INV_SQRT_QK);
    }
    __syncthreads();
    const float qs = qs_s;
    int count, chunk;
    key_chunks_dev(n, nested, &count, &chunk);
    const size_t kvrow = (((size_t)s * c.L + l) * 2 + kvh) * c.cap;
    const int8_t* k8 = c.k8 + kvrow * 48;
    const float* ks = c.ks + kvrow;
    const int8_t* v8 = c.v8 + kvrow * 64;
    const float* vs = c.vs + kvrow;
    int qw4[12];
#pragma unroll
    for (int e = 0; e < 12; e++) qw4[e] = ((const int*)q8)[e];
    for (int ci = 0; ci < count; ci++) {
        const int c0 = ci * chunk, len = min(chunk, n - c0), blocked = len / 4 * 4;
        // scores
        float mx = -INFINITY;
        for (int k = tid; k < len; k += 128) {
            int slot = lo + c0 + k;
            const int* kr = (const int*)(k8 + (size_t)slot * 48);
            int dot = 0;
#pragma unroll
            for (int e = 0; e < 12; e++) dot = __dp4a(qw4[e], kr[e], dot);
            float ksv = ks[slot];
            float sv = k < blocked ? __fmul_rn(__fmul_rn(ksv, (float)dot), qs) : __fmul_rn(__fmul_rn(ksv, qs), (float)dot);
            sbuf[k] = sv;
            mx = fmaxf(mx, sv);
        }
        mx = warp_max(mx);
        if (lane == 0) red[warp] = mx;
        __syncthreads();
        if (tid == 0) m_s = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
        __syncthreads();
        const float mv = m_s;
        // numerators: the inline exp on whole 4-blocks, libm exp after
        const int n4 = len / 4 * 4;
        for (int k = tid; k < len; k += 128) {
            float dlt = __fsub_rn(sbuf[k], mv);
            sbuf[k] = k < n4 ? nexp(dlt) : lexpf(dlt);
        }
        __syncthreads();
        if (tid == 0) {
            // chunk_exp's sum: a[k] over 8-blocks (first halves) and the
            // trailing 4-block, b[k] over the 8-blocks' second halves.
            const int n8 = len / 8 * 8;
            float av[4] = {0.f, 0.f, 0.f, 0.f}, bv[4] = {0.f, 0.f, 0.f, 0.f};
            for (int q = 0; q < n8; q += 8)
                for (int k = 0; k < 4; k++) {
                    av[k] = __fadd_rn(av[k], sbuf[q + k]);
                    bv[k] = __fadd_rn(bv[k], sbuf[q + 4 + k]);
                }
            if (n4 > n8)
                for (int k = 0; k < 4; k++) av[k] = __fadd_rn(av[k], sbuf[n8 + k]);
            float t[4];
            for (int k = 0; k < 4; k++) t[k] = __fadd_rn(av[k], bv[k]);
            float sum = __fadd_rn(__fadd_rn(t[0], t[1]), __fadd_rn(t[2], t[3]));
            int ii = n4;
            if (len - ii >= 2) {
                sum = __fadd_rn(__fadd_rn(sbuf[ii], sum), sbuf[ii + 1]);
                ii += 2;
            }
            if (len - ii == 1) sum = __fadd_rn(sum, sbuf[ii]);
            sum_s = sum;
        }
        __syncthreads();
        // weights times the value scales, their max
        float wm = 0.f;
        for (int k = tid; k < len; k += 128) {
            float wv = __fmul_rn(sbuf[k], vs[lo + c0 + k]);
            sbuf[k] = wv;
            wm = fmaxf(wm, wv);
        }
        wm = warp_max(wm);
        if (lane == 0) red[warp] = wm;
        __syncthreads();
        if (tid == 0) wmax_s = fmaxf(fmaxf(fmaxf(0.f, red[0]), red[1]), fmaxf(red[2], red[3]));
        __syncthreads();
        const float wmax = wmax_s, qw = __fdiv_rn(ND_Q21, wmax);
        for (int k = tid; k < len; k += 128) {
            int wq = (int)roundf(__fmul_rn(sbuf[k], qw));
            dh[k] = (int8_t)(wq >> 14);
            dm_[k] = (int8_t)((wq >> 7) & 127);
            dl[k] = (int8_t)(wq & 127);
        }
        __syncthreads();
        // P.V as three integer dots per value dimension
        {
            const int dm = tid & 63, half = tid >> 6;
            int sh = 0, sm = 0, sl = 0;
            for (int k = half; k < len; k += 2) {
                int v = v8[(size_t)(lo + c0 + k) * 64 + dm];
                sh += dh[k] * v;
                sm += dm_[k] * v;
                sl += dl[k] * v;
            }
            pv[0][half][dm] = sh;
            pv[1][half][dm] = sm;
            pv[2][half][dm] = sl;
        }
        __syncthreads();
        if (tid < 64) {
            int sh = pv[0][0][tid] + pv[0][1][tid], sm = pv[1][0][tid] + pv[1][1][tid], sl = pv[2][0][tid] + pv[2][1][tid];
            float cw = __fmul_rn(wmax, ND_C21);
            po[ci][tid] = __fmul_rn(__fmaf_rn(16384.f, (float)sh, __fmaf_rn(128.f, (float)sm, (float)sl)), cw);
            if (tid == 0) {
                pm[ci] = mv;
                psum[ci] = sum_s;
            }
        }
        __syncthreads();
    }
    if (tid < 64) {
        float out;
        if (count == 1) {
            out = __fmul_rn(po[0][tid], __fdiv_rn(1.0f, psum[0]));
        } else {
            float big = -1e30f;
            for (int ci = 0; ci < count; ci++) big = fmaxf(big, pm[ci]);
            float acc = 0.f, total = 0.f;
            for (int ci = 0; ci < count; ci++) {
                float wv = lexpf(__fsub_rn(pm[ci], big));
                acc = __fmaf_rn(po[ci][tid], wv, acc);
                total = __fmaf_rn(wv, psum[ci], total);
            }
            out = __fmul_rn(acc, __fdiv_rn(1.0f, total));
        }
        float g = proj[(size_t)m * 1568 + 800 + hh * 64 + tid];
        att[(size_t)m * 768 + hh * 64 + tid] = __fdiv_rn(out, __fadd_rn(nexp(-g), 1.0f));
    }
}

void launch_attention(const float* qbuf, const float* proj, Caches c, int l, int S, int T, int p0, int window, float* att,
                      cudaStream_t st) {
    COUNT_LAUNCH();
    attention_kernel<<<dim3(S * T, 12), 128, 0, st>>>(qbuf, proj, c, l, T, p0, window, att);
}

// ------------------------------------------------------------ post block

// infer.rs:1564-1606 with mlp_native (1610-1634), cond_weights (1640-1694),
// kron_native / mix8 (2322-2460), silu (2463-2496), sinkhorn64 (2501-2525).
// One CTA of 1024 threads per row; each Kronecker output is one thread's
// fma chain over j from zero.
__device__ __forceinline__ void kron_stage(const float* z, const float* A, const float* B, float* mt, float* t, int tid) {
    const int r = tid >> 5, cc = tid & 31;
    float o = 0.f;
#pragma unroll 8
    for (int j = 0; j < 32; j++) o = __fmaf_rn(A[j * 32 + r], z[j * 32 + cc], o);
    mt[cc * 33 + r] = o;
    __syncthreads();
    o = 0.f;
#pragma unroll 8
    for (int j = 0; j < 32; j++) o = __fmaf_rn(mt[j * 33 + r], B[j * 32 + cc], o);
    t[r * 32 + cc] = o;
    __syncthreads();
}

__global__ void __launch_bounds__(1024) post_block_kernel(LayerW w, int lane_own, const float* o, const float* x1,
                                                          const float* u, const float* p, const int32_t* perm1,
                                                          const int32_t* perm2, float* xs) {
    __shared__ __align__(16) float x2[768];
    __shared__ __align__(16) float h2[768];
    __shared__ __align__(16) float z[1024];
    __shared__ __align__(16) float t[1024];
    __shared__ float mt[32 * 33];
    __shared__ float part[32];
    __shared__ float sc[2];
    __shared__ float wk[8];
    __shared__ float hpost[4];
    __shared__ float hres[16];
    const int m = blockIdx.x, tid = threadIdx.x;
    if (tid < 768) x2[tid] = o[(size_t)m * 768 + tid];
    __syncthreads();
    if (tid < 16) part[tid] = dot16_chain(x2, x2, 768, tid);
    __syncthreads();
    if (tid == 0) sc[0] = rinv(dot16_combine(part), 768);
    __syncthreads();
    const float ga = __fdiv_rn(1.0f, __fadd_rn(lexpf(-w.attn_gate), 1.0f));
    if (tid < 768) {
        float tt = __fmul_rn(x2[tid], sc[0]);
        float on = __fmaf_rn(tt, w.post_norm[tid], tt);
        x2[tid] = __fmaf_rn(on, ga, x1[(size_t)m * 768 + tid]);
    }
    __syncthreads();
    if (tid < 16) part[tid] = dot16_chain(x2, x2, 768, tid);
    __syncthreads();
    if (tid == 0) sc[1] = rinv(dot16_combine(part), 768);
    __syncthreads();
    if (tid < 768) {
        float tt = __fmul_rn(x2[tid], sc[1]);
        h2[tid] = __fmaf_rn(tt, w.pre_hada[tid], tt);
    }
    __syncthreads();
    // conditioning logits: 4 accumulator sets by j % 4 (fma chains over j)
    if (tid < 32) {
        const int set = tid >> 3, k = tid & 7;
        float acc = 0.f;
        for (int j = set; j < 768; j += 4) acc = __fmaf_rn(h2[j], w.cond_v[j * 8 + k], acc);
        part[tid] = acc;
    }
    __syncthreads();
    if (tid == 0) {
        float lg[8], e[8], mx = -INFINITY;
        for (int k = 0; k < 8; k++) {
            lg[k] = __fadd_rn(__fadd_rn(__fadd_rn(part[16 + k], part[24 + k]), part[8 + k]), part[k]);
            mx = fmaxf(mx, lg[k]);
        }
        for (int k = 0; k < 8; k++) e[k] = lexpf(__fsub_rn(lg[k], mx));
        float sum = __fadd_rn(e[7], __fadd_rn(__fadd_rn(e[6], __fadd_rn(e[5], e[4])), __fadd_rn(__fadd_rn(e[3], e[2]), __fadd_rn(e[1], e[0]))));
        float inv = __fdiv_rn(1.0f, sum);
        for (int k = 0; k < 8; k++) wk[k] = __fmul_rn(e[k], inv);
    }
    z[tid] = tid < 768 ? __fmul_rn(h2[tid], w.d1[tid]) : 0.f;
    __syncthreads();
    kron_stage(z, w.kron[0], w.kron[1], mt, t, tid);
    {
        float cnd = 1.0f;
#pragma unroll
        for (int k = 0; k < 8; k++) cnd = __fmaf_rn(w.cond_u[k * 1024 + tid], wk[k], cnd);
        float zz = __fmaf_rn(t[perm1[tid]], __fmul_rn(cnd, w.d2[tid]), w.b2[tid]);
        z[tid] = __fdiv_rn(zz, __fadd_rn(nexp(-zz), 1.0f));
    }
    __syncthreads();
    kron_stage(z, w.kron[2], w.kron[3], mt, t, tid);
    z[tid] = __fmul_rn(t[perm2[tid]], w.d3[tid]);
    __syncthreads();
    kron_stage(z, w.kron[4], w.kron[5], mt, t, tid);
    if (tid == 0) {
        const float* pr = p + (size_t)m * 24;
        for (int j = 0; j < 4; j++) {
            float off = j == lane_own ? 0.0f : -4.0f;
            float zz = __fadd_rn(__fadd_rn(__fmul_rn(pr[4 + j], w.a_post), off), w.b_post[j]);
            hpost[j] = __fdiv_rn(2.0f, __fadd_rn(lexpf(-zz), 1.0f));
        }
        float zres[16];
        for (int k = 0; k < 16; k++) zres[k] = __fmaf_rn(pr[8 + k], w.a_res, w.b_res[k]);
        double e[16];
        for (int r = 0; r < 4; r++) {
            double mx = (double)fmaxf(fmaxf(zres[r * 4], zres[r * 4 + 1]), fmaxf(zres[r * 4 + 2], zres[r * 4 + 3]));
            for (int cc = 0; cc < 4; cc++) e[r * 4 + cc] = exp(__dsub_rn((double)zres[r * 4 + cc], mx));
        }
        for (int it = 0; it < 20; it++) {
            for (int r = 0; r < 4; r++) {
                double inv = __ddiv_rn(1.0, __dadd_rn(__dadd_rn(e[r * 4], e[r * 4 + 1]), __dadd_rn(e[r * 4 + 2], e[r * 4 + 3])));
                for (int cc = 0; cc < 4; cc++) e[r * 4 + cc] = __dmul_rn(e[r * 4 + cc], inv);
            }
            for (int cc = 0; cc < 4; cc++) {
                double inv = __ddiv_rn(1.0, __dadd_rn(__dadd_rn(e[cc], e[4 + cc]), __dadd_rn(e[8 + cc], e[12 + cc])));
                for (int r = 0; r < 4; r++) e[r * 4 + cc] = __dmul_rn(e[r * 4 + cc], inv);
            }
        }
        for (int k = 0; k < 16; k++) hres[k] = (float)e[k];
    }
    __syncthreads();
    if (tid < 768) {
        const int ch = tid;
        float mlp = __fmul_rn(t[ch], w.d4[ch]);
        float y = __fsub_rn(__fadd_rn(x2[ch], mlp), u[(size_t)m * 768 + ch]);
        float* xr = xs + (size_t)m * 3072;
        float old[4];
#pragma unroll
        for (int b = 0; b < 4; b++) old[b] = xr[b * 768 + ch];
#pragma unroll
        for (int a = 0; a < 4; a++) {
            float v = __fmul_rn(y, hpost[a]);
#pragma unroll
            for (int b = 0; b < 4; b++) v = __fmaf_rn(old[b], hres[a * 4 + b], v);
            xr[a * 768 + ch] = v;
        }
    }
}

void launch_post_block(LayerW w, int lane, const float* o, const float* x1, const float* u, const float* p,
                       const int32_t* perm1, const int32_t* perm2, int M, float* xs, cudaStream_t st) {
    COUNT_LAUNCH();
    post_block_kernel<<<M, 1024, 0, st>>>(w, lane, o, x1, u, p, perm1, perm2, xs);
}

// ------------------------------------------------------------ final norm

// infer.rs:1214-1225: lane mean ((x0 + x1) + x2 + x3) * 0.25, then the final
// ZC-RMSNorm, for each sequence's last row (or every row).
__global__ void final_hidden_kernel(const float* xs, const float* fnorm, int T, int all_rows, float* h) {
    __shared__ float mean[768];
    __shared__ float part[16];
    __shared__ float r_s;
    const int q = blockIdx.x, tid = threadIdx.x;
    const int m = all_rows ? q : q * T + T - 1;
    const float* x = xs + (size_t)m * 3072;
    for (int ch = tid; ch < 768; ch += 256)
        mean[ch] = __fmul_rn(__fadd_rn(__fadd_rn(__fadd_rn(x[ch], x[768 + ch]), x[1536 + ch]), x[2304 + ch]), 0.25f);
    __syncthreads();
    if (tid < 16) part[tid] = dot16_chain(mean, mean, 768, tid);
    __syncthreads();
    if (tid == 0) r_s = rinv(dot16_combine(part), 768);
    __syncthreads();
    for (int ch = tid; ch < 768; ch += 256) {
        float tt = __fmul_rn(mean[ch], r_s);
        h[(size_t)q * 768 + ch] = __fmaf_rn(tt, fnorm[ch], tt);
    }
}

void launch_final_hidden(const float* xs, const float* final_norm, int S, int T, int all_rows, float* h, cudaStream_t st) {
    COUNT_LAUNCH();
    final_hidden_kernel<<<all_rows ? S * T : S, 256, 0, st>>>(xs, final_norm, T, all_rows, h);
}

// ----------------------------------------------------------------- RoPE

// infer.rs:1716-1744: table rows (sincosf of freq * pos, tabulated on the
// host with the reference's f64 libm stand-in) for a chunk, or for a single
// token right after the newest position the angle-addition recurrence.
__global__ void rope_rows_kernel(const float* tc, const float* tsn, const float* sd, const float* cd, int p0, int T, int recur,
                                 float* state, float* cosr, float* sinr) {
    int i = blockIdx.x, f = threadIdx.x;
    if (f >= 24) return;
    float cv, sv;
    if (recur) {
        float c0 = state[f], s0 = state[24 + f];
        cv = __fmaf_rn(-sd[f], s0, __fmul_rn(cd[f], c0));
        sv = __fmaf_rn(sd[f], c0, __fmul_rn(cd[f], s0));
    } else {
        cv = tc[(size_t)(p0 + i) * 24 + f];
        sv = tsn[(size_t)(p0 + i) * 24 + f];
    }
    cosr[i * 24 + f] = cv;
    sinr[i * 24 + f] = sv;
    if (i == T - 1) {
        state[f] = cv;
        state[24 + f] = sv;
    }
}

void launch_rope_rows(const float* table_cos, const float* table_sin, const float* sd, const float* cd, int p0, int T,
                      int recur, float* state, float* cosr, float* sinr, cudaStream_t st) {
    COUNT_LAUNCH();
    rope_rows_kernel<<<T, 32, 0, st>>>(table_cos, table_sin, sd, cd, p0, T, recur, state, cosr, sinr);
}

// ------------------------------------------------------- masked argmax

// crates/needle-engine/src/agent.rs:1114-1127: banned ids read -1e30, then
// the first index of the maximum.
__global__ void masked_argmax_kernel(const float* logits, int V, const uint8_t* allow, int32_t* next) {
    __shared__ float bv[32];
    __shared__ int bi[32];
    const int s = blockIdx.x, tid = threadIdx.x;
    const float* x = logits + (size_t)s * V;
    const uint8_t* al = allow ? allow + (size_t)s * ((V + 7) / 8) : nullptr;
    float best = -INFINITY;
    int idx = 0x7fffffff;
    for (int k = tid; k < V; k += blockDim.x) {
        float v = (!al || ((al[k >> 3] >> (k & 7)) & 1)) ? x[k] : -1e30f;
        if (v > best || (v == best && k < idx)) { best = v; idx = k; }
    }
    for (int o = 16; o; o >>= 1) {
        float ov = __shfl_xor_sync(0xffffffffu, best, o);
        int oi = __shfl_xor_sync(0xffffffffu, idx, o);
        if (ov > best || (ov == best && oi < idx)) { best = ov; idx = oi; }
    }
    if ((tid & 31) == 0) { bv[tid >> 5] = best; bi[tid >> 5] = idx; }
    __syncthreads();
    if (tid == 0) {
        int nw = blockDim.x >> 5;
        for (int k = 1; k < nw; k++)
            if (bv[k] > best || (bv[k] == best && bi[k] < idx)) { best = bv[k]; idx = bi[k]; }
        next[s] = idx == 0x7fffffff ? 0 : idx;
    }
}

void launch_masked_argmax(const float* logits, int S, int V, const uint8_t* allow, int32_t* next, cudaStream_t st) {
    COUNT_LAUNCH();
    masked_argmax_kernel<<<S, 1024, 0, st>>>(logits, V, allow, next);
}

}  // namespace nd
