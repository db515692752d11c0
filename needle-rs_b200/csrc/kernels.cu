// Kernels of the Needle 3 packed forward pass (sm_100a).
//
// Each kernel reproduces one phase of the reference's native path
// (crates/needle-engine/src/infer.rs `chunk_native`/`layer_native`) for every
// row of a step at once. Integer sums are exact, so their order is free; every
// float op follows the reference's order, rounding and fusion.

#include <algorithm>
#include <utility>
#include <atomic>

#include "kernels.h"
#include "numerics.cuh"
#include "cqrow.cuh"

namespace nd {

// Programmatic dependent launch: every kernel here is launched so that the
// next kernel of its stream may start once all of this one's CTAs have
// started (pdl_launch_dependents), and waits for its predecessor's results
// (pdl_wait: the predecessor grid has completed and its writes are visible)
// before touching anything the predecessor reads or writes.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory"); }

template <typename... KArgs, typename... Args>
static void launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args&&... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = st ? 1 : 0;  // the legacy default stream keeps plain ordering
    cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}


static std::atomic<long long> g_launches{0};
long long launch_count() { return g_launches.load(); }
void add_launches(long long n) { g_launches.fetch_add(n, std::memory_order_relaxed); }
#define COUNT_LAUNCH() g_launches.fetch_add(1, std::memory_order_relaxed)

__constant__ float c_hs128;       // (float)(1/sqrt(128)), quant.rs:71-73

static cudaError_t init_attrs();

void set_constants(float hs128) {
    init_attrs();
    cudaMemcpyToSymbol(c_hs128, &hs128, 4);
}

static inline int cdiv(int a, int b) { return (a + b - 1) / b; }

// SM count of the current device, looked up once per device id. Launchers
// run on any host thread, so the cache is atomic: two threads that both
// miss store the same value.
static int sm_count() {
    static std::atomic<int> sms[64];
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return 148;
    int v = sms[dev].load(std::memory_order_relaxed);
    if (!v) {
        if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0) v = 148;
        sms[dev].store(v, std::memory_order_relaxed);
    }
    return v;
}

int device_sm_count() { return sm_count(); }

// --------------------------------------------------------------- tokens

__global__ void write_tokens_kernel(const int32_t* ids, int S, int T, const int32_t* p0p, int32_t* tokens, int cap) {
    pdl_launch_dependents();
    pdl_wait();
    const int p0 = *p0p;
    int m = blockIdx.x * blockDim.x + threadIdx.x;
    if (m >= S * T) return;
    int s = m / T, i = m % T;
    tokens[(size_t)s * cap + p0 + i] = ids[m];
}

void launch_write_tokens(const int32_t* ids, int S, int T, int p0, Caches c, cudaStream_t st) {
    COUNT_LAUNCH();
    launch_pdl(write_tokens_kernel, dim3(cdiv(S * T, 256)), dim3(256), 0, st, ids, S, T, c.len, c.tokens, c.cap);
}

// ------------------------------------------------------- CQ row dequant

// infer.rs:1185-1194: the embedding row times sqrt(d), in every lane.
__global__ void embed_kernel(DevMat emb, const int32_t* ids, float* xs, float scale) {
    pdl_launch_dependents();
    pdl_wait();
    int m = blockIdx.x, g = blockIdx.y, lane = threadIdx.x;
    int tok = ids[m];
    float v[4];
    cq_group_row(emb, (size_t)tok, g, lane, v);
    float4 o = make_float4(__fmul_rn(v[0], scale), __fmul_rn(v[1], scale), __fmul_rn(v[2], scale), __fmul_rn(v[3], scale));
    const int d = emb.in_dim;
#pragma unroll
    for (int ln = 0; ln < 4; ln++) *(float4*)(xs + (size_t)m * 4 * d + ln * d + g * 128 + 4 * lane) = o;
}

void launch_embed(DevMat emb, const int32_t* ids, int M, float* xs, cudaStream_t st) {
    COUNT_LAUNCH();
    float scale = __builtin_sqrtf((float)emb.in_dim);
    launch_pdl(embed_kernel, dim3(dim3(M, emb.groups)), dim3(32), 0, st, emb, ids, xs, scale);
}

// ------------------------------------------------------------ A8 prep

// prep_group (qlinear.rs:152-164): zero-pad, rotate, int8 with one scale per
// (row, group). Stored lane-major: input p = 32a + 8l + b of a group (a, l <
// 4, b < 8) sits at slot l*32 + (a&1)*16 + (a>>1)*8 + b. Both decode lane
// rules of qlinear.rs:333 are then 16-byte aligned runs of slots: the 4-bit
// lane (p % 32) / 8 = l is the 32 bytes l*32 .., and the 2-bit lane
// (p % 64) / 16 = 2(a&1) + (l>>1) the two 16-byte halves at
// (2(lane&1) + h)*32 + (lane>>1)*16, h = 0, 1. The weights' w8 copy uses the
// same slots, so any run of slots meets its own inputs. Warp lane i holds
// p = 4i .. 4i + 3.
__host__ __device__ __forceinline__ int lane_major_slot_of(int p) {
    const int a = p >> 5, l = (p >> 3) & 3, b = p & 7;
    return l * 32 + (a & 1) * 16 + (a >> 1) * 8 + b;
}
__device__ __forceinline__ int lane_major_pos(int i) { return lane_major_slot_of(4 * i); }
int lane_major_slot(int p) { return lane_major_slot_of(p); }

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
    *(char4*)(q + lane_major_pos(lane)) = o;
    if (lane == 0) *sx = s;
}

__global__ void prep_act_kernel(const float* x, int ldx, int K, int8_t* act, float* sx, int G) {
    pdl_launch_dependents();
    pdl_wait();
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
    launch_pdl(prep_act_kernel, dim3(dim3(M, G)), dim3(32), 0, st, x, ldx, K, act, sx, G);
}

// ----------------------------------------------------------- CQ matmul

// The decode combine (qlinear.rs:340-350) for T == 1: four float lanes per
// output, lane l fed by inputs p with (p % 32) / 8 == l (width 2: (p % 64)
// / 16 == l), scale (sx * cbs) * norm, lanes summed (l0 + l1) + (l2 + l3). The prefill
// combine (qlinear.rs:353-363) otherwise: one fma chain over groups, scale
// (norm * cbs) * sx for a sequence's first T/4*4 rows, norm * (cbs * sx)
// for the rest.

// ---------------------------------------------- CQ matmul on tensor cores
//
// The two combines with the integer sums from mma.sync m16n8k32 s8: with
// both operands lane-major, decode lane l of group g is two 16-byte runs of
// the K axis (the A and B fragments' halves), so one MMA gives exactly one
// lane sum (decode) and four chained MMAs one group sum (prefill). Each accumulator starts at the bit
// pattern of 1.5 * 2^23: every sum here is below 2^22 in magnitude, so the
// result reinterpreted as a float minus 1.5 * 2^23 is the sum, exactly, in
// one FP32 subtract. CTA tile 64 rows x 64 outputs, K = 768 resident in
// shared memory, loaded one 128-wide group at a time with cp.async so the
// first groups compute while the rest arrive.
constexpr int MMA_BM = 64, MMA_BN = 64, MMA_K = 768, MMA_LD = MMA_K + 16;
constexpr int MMA_MAGIC = 0x4B400000;
constexpr size_t MMA_SMEM = (size_t)(MMA_BM + MMA_BN) * MMA_LD + (size_t)2 * MMA_BM * 6 * 4 + (size_t)2 * MMA_BN * 6 * 2;

__device__ __forceinline__ void mma_s8(int (&d)[4], const uint32_t (&a)[4], const uint32_t (&b)[2], const int (&c)[4]) {
    asm(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%11,%12,%13};\n"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]), "r"(c[0]), "r"(c[1]), "r"(c[2]), "r"(c[3]));
}

// Four 8x8 b16 matrices (8 rows of 16 bytes each); lanes 8q..8q+7 give
// matrix q's row addresses, and lane t receives row t / 4, bytes
// 4 (t % 4) .. 4 (t % 4) + 3 of each, in r[q]: the int8 mma fragments.
__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
    uint32_t s = (uint32_t)__cvta_generic_to_shared(p);
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(s)
                 : "memory");
}

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool valid) {
    uint32_t s = (uint32_t)__cvta_generic_to_shared(smem);
    int n = valid ? 16 : 0;
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(s), "l"(gmem), "r"(n));
}

__device__ __forceinline__ void cp_async4(void* smem, const void* gmem) {
    uint32_t s = (uint32_t)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(s), "l"(gmem));
}

// fma.rn.f32x2: two independent IEEE fmas in one instruction (sm_100).
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) {
    float2 d;
    asm("{\n.reg .b64 ra, rb, rc, rd;\nmov.b64 ra, {%2, %3};\nmov.b64 rb, {%4, %5};\nmov.b64 rc, {%6, %7};\n"
        "fma.rn.f32x2 rd, ra, rb, rc;\nmov.b64 {%0, %1}, rd;\n}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
    return d;
}

// add.rn.f32x2 / sub.rn.f32x2: two independent IEEE adds (subtractions).
__device__ __forceinline__ float2 add2(float2 a, float2 b) {
    float2 d;
    asm("{\n.reg .b64 ra, rb, rd;\nmov.b64 ra, {%2, %3};\nmov.b64 rb, {%4, %5};\n"
        "add.rn.f32x2 rd, ra, rb;\nmov.b64 {%0, %1}, rd;\n}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return d;
}

__device__ __forceinline__ float2 sub2(float2 a, float2 b) {
    float2 d;
    asm("{\n.reg .b64 ra, rb, rd;\nmov.b64 ra, {%2, %3};\nmov.b64 rb, {%4, %5};\n"
        "sub.rn.f32x2 rd, ra, rb;\nmov.b64 {%0, %1}, rd;\n}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return d;
}

// The decode lane update for two adjacent outputs of one mma: the two int32
// sums (accumulated from the magic 1.5 * 2^23) become floats with one
// paired subtraction and join their lane chains with one paired fma. The
// pairs stay packed in 64-bit registers.
__device__ __forceinline__ void lane_fma2(unsigned long long& acc, int d0, int d1, unsigned long long sc) {
    const unsigned long long mg = 0x4B4000004B400000ull;  // 12582912.0f twice
    asm("{\n.reg .b64 x;\nmov.b64 x, {%1, %2};\nsub.rn.f32x2 x, x, %4;\nfma.rn.f32x2 %0, x, %3, %0;\n}"
        : "+l"(acc)
        : "r"(d0), "r"(d1), "l"(sc), "l"(mg));
}

__device__ __forceinline__ unsigned long long pack2(float a, float b) {
    return (unsigned long long)__float_as_uint(a) | ((unsigned long long)__float_as_uint(b) << 32);
}

__device__ __forceinline__ float2 unpack2(unsigned long long v) {
    return make_float2(__uint_as_float((unsigned)v), __uint_as_float((unsigned)(v >> 32)));
}

__device__ __forceinline__ float magic_to_float(int v) { return __fsub_rn(__int_as_float(v), 12582912.0f); }

__device__ __forceinline__ void cp_async4z(void* smem, const void* gmem, bool valid) {
    uint32_t s = (uint32_t)__cvta_generic_to_shared(smem);
    int n = valid ? 4 : 0;
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;\n" ::"r"(s), "l"(gmem), "r"(n));
}

// Persistent: CTA b takes tiles b, b + grid, ... (n-tile fastest). Its
// iterations k run group k % 6 of tile k / 6; the copies of iteration k + 5
// are issued at iteration k into the slot iteration k - 1 has just freed, so
// the next tile's operands arrive while this one computes. A tile's scales
// (activation sx, f16 norms) come with its group 0 into one of two buffers.
// K offset within a group of half h of decode lane l (lane_major_pos).
template <bool TWO>
__device__ __forceinline__ int lane_half(int l, int h) {
    return TWO ? (2 * (l & 1) + h) * 32 + (l >> 1) * 16 : l * 32 + h * 16;
}

template <bool DECODE, bool TWO>
__global__ void __launch_bounds__(256, 2) cq_mma_kernel(DevMat W, const int8_t* act, const float* sx, int M, int T, float* y,
                                                        int ldy, int col0) {
    pdl_launch_dependents();
    extern __shared__ __align__(16) int8_t smem[];
    int8_t* ws = smem;                                        // [BN][LD]
    int8_t* as = smem + MMA_BN * MMA_LD;                      // [BM][LD]
    float* s_sx = (float*)(as + MMA_BM * MMA_LD);             // [2][BM][6]
    uint16_t* s_nr = (uint16_t*)(s_sx + 2 * MMA_BM * 6);      // [2][BN][6] f16
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int tilesN = (W.out + MMA_BN - 1) / MMA_BN, ntiles = tilesN * ((M + MMA_BM - 1) / MMA_BM);
    const int first = blockIdx.x, stride = gridDim.x;
    const int iters = first < ntiles ? ((ntiles - 1 - first) / stride + 1) * 6 : 0;
    // the copies of iteration k: the weight rows (and the tile's norms) when
    // W, the activation rows (and their scales) when A
    auto issue_part = [&](int k, bool wpart, bool apart) {
        if (k < iters) {
            const int t = first + (k / 6) * stride, g = k % 6;
            const int tn0 = (t % tilesN) * MMA_BN, tm0 = (t / tilesN) * MMA_BM;
            for (int idx = tid; idx < (MMA_BN + MMA_BM) * 8; idx += 256) {
                int r = idx >> 3, c = idx & 7;
                if (r < MMA_BN) {
                    int n = tn0 + r;
                    bool ok = n < W.out;
                    if (wpart)
                        cp_async16(ws + r * MMA_LD + g * 128 + c * 16, W.w8 + (size_t)(ok ? n : 0) * MMA_K + g * 128 + c * 16, ok);
                } else {
                    int mr = r - MMA_BN, m = tm0 + mr;
                    bool ok = m < M;
                    if (apart)
                        cp_async16(as + mr * MMA_LD + g * 128 + c * 16, act + (size_t)(ok ? m : 0) * MMA_K + g * 128 + c * 16, ok);
                }
            }
            if (g == 0) {
                float* bx = s_sx + ((k / 6) & 1) * MMA_BM * 6;
                uint16_t* bn = s_nr + ((k / 6) & 1) * MMA_BN * 6;
                if (apart)
                    for (int idx = tid; idx < MMA_BM * 6; idx += 256) {
                        const int m = tm0 + idx / 6;
                        cp_async4z(bx + idx, sx + (size_t)(m < M ? m : 0) * 6 + idx % 6, m < M);
                    }
                if (wpart)
                    for (int idx = tid; idx < MMA_BN * 3; idx += 256) {
                        const int n = tn0 + idx / 3;
                        cp_async4z(bn + 2 * idx, W.norms + (size_t)(n < W.out ? n : 0) * 6 + 2 * (idx % 3), n < W.out);
                    }
            }
        }
    };
    auto issue = [&](int k) {
        issue_part(k, true, true);
        asm volatile("cp.async.commit_group;\n" ::);
    };
    // the first five iterations' weight copies go out before the wait on the
    // predecessor (they join the first commit group), their activation
    // copies after it, one commit group each
#pragma unroll 1
    for (int k = 0; k < 5; k++) issue_part(k, true, false);
    pdl_wait();
#pragma unroll 1
    for (int k = 0; k < 5; k++) {
        issue_part(k, false, true);
        asm volatile("cp.async.commit_group;\n" ::);
    }
    const float cbs = W.cbs;
    const int wm = (warp & 3) * 16, wn = (warp >> 2) * 32;
    const int gid = lane >> 2, tig = lane & 3;
    const int r0 = wm + gid, r1 = r0 + 8;  // this thread's two rows in the tile
    float acc[4][4];       // prefill: [n-tile][element]
    unsigned long long accd[4][2][4];  // decode: [n-tile][row pair][lane], adjacent columns packed
#pragma unroll
    for (int j = 0; j < 4; j++) {
#pragma unroll
        for (int e = 0; e < 4; e++) acc[j][e] = 0.f;
#pragma unroll
        for (int pp = 0; pp < 2; pp++)
#pragma unroll
            for (int l = 0; l < 4; l++) accd[j][pp][l] = 0ull;
    }
    const int magic[4] = {MMA_MAGIC, MMA_MAGIC, MMA_MAGIC, MMA_MAGIC};
    int n0 = 0, m0 = 0;
    bool blk0 = true, blk1 = true;  // prefill: block rows t < T/4*4
    const float* tsx = s_sx;
    const uint16_t* tnr = s_nr;
#pragma unroll 1
    for (int k = 0; k < iters; k++) {
        const int g = k % 6;
        asm volatile("cp.async.wait_group 4;\n" ::);
        __syncthreads();
        issue(k + 5);
        if (g == 0) {
            const int t = first + (k / 6) * stride;
            n0 = (t % tilesN) * MMA_BN;
            m0 = (t / tilesN) * MMA_BM;
            tsx = s_sx + ((k / 6) & 1) * MMA_BM * 6;
            tnr = s_nr + ((k / 6) & 1) * MMA_BN * 6;
            if (!DECODE) {
                blk0 = ((m0 + r0) % T) < T / 4 * 4;
                blk1 = ((m0 + r1) % T) < T / 4 * 4;
            }
        }
        // scales of this group for this thread's rows and columns
        float rs0, rs1, cs[4][2];
        if (DECODE) {
            rs0 = __fmul_rn(tsx[r0 * 6 + g], cbs);
            rs1 = __fmul_rn(tsx[r1 * 6 + g], cbs);
        } else {
            rs0 = blk0 ? tsx[r0 * 6 + g] : __fmul_rn(tsx[r0 * 6 + g], cbs);
            rs1 = blk1 ? tsx[r1 * 6 + g] : __fmul_rn(tsx[r1 * 6 + g], cbs);
        }
#pragma unroll
        for (int j = 0; j < 4; j++)
#pragma unroll
            for (int h = 0; h < 2; h++) cs[j][h] = h2f(tnr[(wn + j * 8 + tig * 2 + h) * 6 + g]);
        // decode: (sx * cbs) * norm for each of this thread's outputs, as
        // pairs of adjacent columns
        unsigned long long dsc[4][2];
        if (DECODE) {
#pragma unroll
            for (int j = 0; j < 4; j++)
#pragma unroll
                for (int pp = 0; pp < 2; pp++)
                    dsc[j][pp] = pack2(__fmul_rn(pp ? rs1 : rs0, cs[j][0]), __fmul_rn(pp ? rs1 : rs0, cs[j][1]));
        }
        int dsum[4][4];
#pragma unroll
        for (int l = 0; l < 4; l++) {
            uint32_t a[4], bq[2][4];
            ldsm_x4(a, as + (wm + (lane & 15)) * MMA_LD + g * 128 + lane_half<TWO>(l, lane >> 4));
#pragma unroll
            for (int jj = 0; jj < 2; jj++)
                ldsm_x4(bq[jj], ws + (wn + (2 * jj + (lane >> 4)) * 8 + (lane & 7)) * MMA_LD + g * 128 +
                                    lane_half<TWO>(l, (lane >> 3) & 1));
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const uint32_t b[2] = {bq[j >> 1][(j & 1) * 2], bq[j >> 1][(j & 1) * 2 + 1]};
                int d[4];
                if (DECODE) {
                    mma_s8(d, a, b, magic);
                    lane_fma2(accd[j][0][l], d[0], d[1], dsc[j][0]);
                    lane_fma2(accd[j][1][l], d[2], d[3], dsc[j][1]);
                } else {
                    if (l == 0) {
                        mma_s8(d, a, b, magic);
                    } else {
                        int c[4] = {dsum[j][0], dsum[j][1], dsum[j][2], dsum[j][3]};
                        mma_s8(d, a, b, c);
                    }
#pragma unroll
                    for (int e = 0; e < 4; e++) dsum[j][e] = d[e];
                }
            }
        }
        if (!DECODE) {
#pragma unroll
            for (int j = 0; j < 4; j++)
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    const bool blk = e < 2 ? blk0 : blk1;
                    // block rows: (norm * cbs) * sx; remainder rows: norm * (cbs * sx)
                    float sc = blk ? __fmul_rn(__fmul_rn(cs[j][e & 1], cbs), e < 2 ? rs0 : rs1)
                                   : __fmul_rn(cs[j][e & 1], e < 2 ? rs0 : rs1);
                    acc[j][e] = __fmaf_rn(magic_to_float(dsum[j][e]), sc, acc[j][e]);
                }
        }
        if (g == 5) {
#pragma unroll
            for (int j = 0; j < 4; j++)
#pragma unroll
                for (int pp = 0; pp < 2; pp++) {
                    // decode: the lanes summed (l0 + l1) + (l2 + l3)
                    float2 v = DECODE ? add2(add2(unpack2(accd[j][pp][0]), unpack2(accd[j][pp][1])),
                                             add2(unpack2(accd[j][pp][2]), unpack2(accd[j][pp][3])))
                                      : make_float2(acc[j][2 * pp], acc[j][2 * pp + 1]);
                    const int m = m0 + (pp ? r1 : r0), n = n0 + wn + j * 8 + tig * 2;
                    if (m < M) {
                        if (n < W.out) y[(size_t)m * ldy + col0 + n] = v.x;
                        if (n + 1 < W.out) y[(size_t)m * ldy + col0 + n + 1] = v.y;
                    }
#pragma unroll
                    for (int l = 0; l < 4; l++) accd[j][pp][l] = 0ull;
                    acc[j][2 * pp] = acc[j][2 * pp + 1] = 0.f;
                }
        }
    }
}

// ------------------------------------------------ CQ matvec (decode, few rows)
//
// The decode combine for one to four activation rows straight off the
// codes, one warp per output row. A group is 16 blocks of 8 inputs (block w
// = inputs p = 8w .. 8w + 7, a = w / 4, l = w % 4 in lane_major_pos's
// terms); lane i holds blocks i, i + 32 and i + 64 of the row (group g = 2k
// + i/16, block i % 16). A block's eight codes (a 32-bit word at 4 bits, a
// 16-bit one at 2 bits) become int8 codebook values with byte permutes, and
// meet their eight lane-major activation bytes in two dp4a; width 3 reads
// the block from the expanded w8 copy instead. Xor-shuffles over the blocks
// of one decode lane give each (group, lane) sum: for the 4-bit rule the
// blocks of lane l are i % 16 = l + 4a (xor 4, 8), for the 2-bit rule
// (p % 64) / 16 = 2(a&1) + (l>>1) they are i % 16 = 2 lane + {0, 1, 8, 9}
// (xor 1, 8). Lanes 0-3 then run the reference's fma chain over groups.
constexpr int GEMV_MAXM = 4;
// From this many one-token rows the decode combine runs on the tensor-core
// kernel (tc_prefill.cu); between GEMV_MAXM and it, on int8 mma.sync tiles.
// The prefill combine likewise from TC_PREFILL_MIN_ROWS rows (a few chunks of
// 32: below that the tensor-core kernel has too few tiles to fill the GPU).
constexpr int TC_DECODE_MIN_ROWS = 64;
constexpr int TC_PREFILL_MIN_ROWS = 256;

__device__ __forceinline__ uint32_t lut4(uint32_t nib16, uint32_t v0, uint32_t v1, uint32_t v2, uint32_t v3) {
    uint32_t idx = nib16 & 0x7777u;
    uint32_t lo = __byte_perm(v0, v1, idx), hi = __byte_perm(v2, v3, idx);
    return __byte_perm(lo, hi, 0x3210u | ((nib16 & 0x8888u) >> 1));
}

// Four 2-bit codes (one byte) through the 4-entry table v.
__device__ __forceinline__ uint32_t lut2(uint32_t c, uint32_t v) {
    const uint32_t sel = (c & 3u) | ((c & 0xCu) << 2) | ((c & 0x30u) << 4) | ((c & 0xC0u) << 6);
    return __byte_perm(v, 0u, sel);
}

// One weight row of the GEMV as a warp holds it: lane i's three blocks
// (codes turned into int8 codebook values) and, in lanes g < 6, the row's
// group norms.
struct GemvRow {
    int wl[3], wh[3];
    float norm_l;
};

// FMT: 4 or 2 = codes of that width, 8 = the w8 copy (width 3). The load
// reads and decodes weight row n (the layer's, not a predecessor's output:
// callers issue it before their wait on the predecessor).
template <int FMT>
__device__ __forceinline__ void gemv_row_load(const DevMat& W, int n, int lane, GemvRow& r) {
    const int wi = lane & 15, a = wi >> 2, l = wi & 3, half = lane >> 4;
    const int slot = l * 32 + (a & 1) * 16 + (a >> 1) * 8;  // lane_major_pos of the block
    if (FMT == 4) {
        const uint32_t v0 = W.vals4[0], v1 = W.vals4[1], v2 = W.vals4[2], v3 = W.vals4[3];
        const uint32_t* codes = (const uint32_t*)(W.codes + (size_t)n * 384);
#pragma unroll
        for (int k = 0; k < 3; k++) {
            const uint32_t c = __ldg(codes + lane + 32 * k);
            r.wl[k] = (int)lut4(c & 0xffffu, v0, v1, v2, v3);
            r.wh[k] = (int)lut4(c >> 16, v0, v1, v2, v3);
        }
    } else if (FMT == 2) {
        const uint32_t v0 = W.vals4[0];
        const uint16_t* codes = (const uint16_t*)(W.codes + (size_t)n * 192);
#pragma unroll
        for (int k = 0; k < 3; k++) {
            const uint32_t c = __ldg(codes + lane + 32 * k);
            r.wl[k] = (int)lut2(c & 0xffu, v0);
            r.wh[k] = (int)lut2(c >> 8, v0);
        }
    } else {
#pragma unroll
        for (int k = 0; k < 3; k++) {
            const int2 w = __ldg((const int2*)(W.w8 + (size_t)n * 768 + (2 * k + half) * 128 + slot));
            r.wl[k] = w.x;
            r.wh[k] = w.y;
        }
    }
    r.norm_l = lane < 6 ? h2f(W.norms[(size_t)n * 6 + lane]) : 0.f;
}

// The decode combine of a loaded row against M activation rows: y[m][col0 + n].
template <int FMT>
__device__ __forceinline__ void gemv_row_out(const DevMat& W, const GemvRow& r, int n, int lane, const int8_t* act, const float* sx,
                                             int M, float* y, int ldy, int col0) {
    const int wi = lane & 15, a = wi >> 2, l = wi & 3, half = lane >> 4;
    const int slot = l * 32 + (a & 1) * 16 + (a >> 1) * 8;
    const float cbs = W.cbs;
    for (int m = 0; m < M; m++) {
        const int8_t* ar = act + (size_t)m * 768;
        int s[3];
#pragma unroll
        for (int k = 0; k < 3; k++) {
            const int g = 2 * k + half;
            const int2 x = *(const int2*)(ar + g * 128 + slot);
            int v = __dp4a(r.wl[k], x.x, 0);
            v = __dp4a(r.wh[k], x.y, v);
            v += __shfl_xor_sync(0xffffffffu, v, FMT == 2 ? 1 : 4);
            v += __shfl_xor_sync(0xffffffffu, v, 8);
            s[k] = v;  // the sum of group g, one decode lane
        }
        float sxl = lane < 6 ? sx[(size_t)m * 6 + lane] : 0.f;
        float acc = 0.f;
#pragma unroll
        for (int g = 0; g < 6; g++) {
            const int src = (g & 1) * 16 + (FMT == 2 ? 2 * (lane & 3) : (lane & 3));
            int sg = __shfl_sync(0xffffffffu, s[g >> 1], src);
            float sc = __fmul_rn(__fmul_rn(__shfl_sync(0xffffffffu, sxl, g), cbs), __shfl_sync(0xffffffffu, r.norm_l, g));
            acc = __fmaf_rn((float)sg, sc, acc);
        }
        float l1 = __shfl_sync(0xffffffffu, acc, 1), l2 = __shfl_sync(0xffffffffu, acc, 2), l3 = __shfl_sync(0xffffffffu, acc, 3);
        if (lane == 0) y[(size_t)m * ldy + col0 + n] = __fadd_rn(__fadd_rn(acc, l1), __fadd_rn(l2, l3));
    }
}

template <int FMT>
__global__ void __launch_bounds__(256) cq_gemv_kernel(DevMat W, const int8_t* act, const float* sx, int M, float* y, int ldy,
                                                      int col0) {
    pdl_launch_dependents();
    // the weight row's codes and norms are the layer's, not the predecessor's:
    // they are read and decoded before the wait on it
    const int lane = threadIdx.x & 31;
    const int n = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (n >= W.out) {
        pdl_wait();
        return;
    }
    GemvRow r;
    gemv_row_load<FMT>(W, n, lane, r);
    pdl_wait();
    gemv_row_out<FMT>(W, r, n, lane, act, sx, M, y, ldy, col0);
}

cudaError_t launch_cq_gemm(DevMat W, const int8_t* act, const float* sx, int M, int T, float* y, int ldy, int col0,
                           cudaStream_t st) {
    if (!W.w8 || W.groups != 6 || W.in_dim != 768 || (W.width != 2 && W.width != 3 && W.width != 4))
        return cudaErrorInvalidValue;  // every matmul here reads 768 inputs, w8 expanded
    COUNT_LAUNCH();
    if (T == 1 && M <= GEMV_MAXM) {
        const dim3 grid(cdiv(W.out, 8));
        if (W.width == 4) launch_pdl(cq_gemv_kernel<4>, grid, dim3(256), 0, st, W, act, sx, M, y, ldy, col0);
        else if (W.width == 2) launch_pdl(cq_gemv_kernel<2>, grid, dim3(256), 0, st, W, act, sx, M, y, ldy, col0);
        else launch_pdl(cq_gemv_kernel<8>, grid, dim3(256), 0, st, W, act, sx, M, y, ldy, col0);
        return cudaSuccess;
    }
    if (T > 1 && M >= TC_PREFILL_MIN_ROWS) return launch_cq_prefill_tc(W, act, sx, M, T, y, ldy, col0, st);
    if (T == 1 && M >= TC_DECODE_MIN_ROWS && W.width != 2) return launch_cq_decode_tc(W, act, sx, M, y, ldy, col0, st);
    const int per = 2 * sm_count();
    const int grid = std::min(cdiv(W.out, MMA_BN) * cdiv(M, MMA_BM), per);
    if (T > 1)
        launch_pdl(cq_mma_kernel<false, false>, dim3(grid), dim3(256), MMA_SMEM, st, W, act, sx, M, T, y, ldy, col0);
    else if (W.width == 2)
        launch_pdl(cq_mma_kernel<true, true>, dim3(grid), dim3(256), MMA_SMEM, st, W, act, sx, M, T, y, ldy, col0);
    else
        launch_pdl(cq_mma_kernel<true, false>, dim3(grid), dim3(256), MMA_SMEM, st, W, act, sx, M, T, y, ldy, col0);
    return cudaSuccess;
}


extern const size_t ATT_SMEM;
extern const size_t POST_ROW_SMEM;
__global__ void post_row_kernel(LayerW w, const float* o, const float* x1, const float* u, const float* gates, const int32_t* perm1,
                                const int32_t* perm2, float* xs);
cudaError_t post_block_init();
template <int MINB>
__global__ void attention_kernel(const float* qbuf, const float* proj, Caches c, int l, int T, const int32_t* p0p, int window,
                                 int sink, int ring, float* att, int8_t* act, float* sx);


// ---------------------------------------------------------------- engram

// infer.rs:1257-1277: the n-gram hash of each (order, head) picks a table
// row; rows the position is too young for stay zero.
__global__ void engram_gather_kernel(DevMat tables, const int32_t* tokens, int cap, int T, const int32_t* p0p, int slots, float* e) {
    pdl_launch_dependents();
    pdl_wait();
    const int p0 = *p0p;
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
        cq_group_row(tables, row, 0, lane, v);
    }
    *(float4*)(e + (size_t)m * d + tbl * sub + 4 * lane) = make_float4(v[0], v[1], v[2], v[3]);
}

void launch_engram_gather(DevMat tables, Caches c, int S, int T, int p0, int slots, float* e, cudaStream_t st) {
    COUNT_LAUNCH();
    launch_pdl(engram_gather_kernel, dim3(dim3(S * T, 6)), dim3(32), 0, st, tables, c.tokens, c.cap, T, c.len, slots, e);
}

// infer.rs:1283-1303: the value half of kv, int8 in 32-wide groups, into
// the site's history at the row's position.
__global__ void engram_vhist_kernel(const float* kv, int8_t* ev8, float* evs, int site, int nsites, int T, const int32_t* p0p) {
    pdl_launch_dependents();
    pdl_wait();
    const int p0 = *p0p;
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
    launch_pdl(engram_vhist_kernel, dim3(S * T), dim3(768), 0, st, kv, c.ev8, c.evs, site, nsites, T, c.len);
}

// infer.rs:1310-1323 with engram_tap (663-687): four taps at dilation 3,
// each an fma from the int8 history.
__global__ void engram_conv_kernel(const float* taps, const int8_t* ev8, const float* evs, int site, int nsites, int T, const int32_t* p0p,
                                   float* v) {
    pdl_launch_dependents();
    pdl_wait();
    const int p0 = *p0p;
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
    launch_pdl(engram_conv_kernel, dim3(S * T), dim3(768), 0, st, taps, c.ev8, c.evs, site, nsites, T, c.len, v);
}

// ------------------------------------------------------------ mHC read

// The mHC read CTA: its six warps (192 threads) each own 16 consecutive
// elements of the row's 3072 per thread; afterwards warp 5 stores the post
// block's gate projections while warps 0-4 (160 threads) run the input
// norm, synchronising among themselves with a named barrier.
constexpr int MHC_THREADS = 192, MHC_NORM_THREADS = 160, MHC_XS = 196;
__device__ __forceinline__ void norm_bar() { asm volatile("bar.sync 1, 160;\n" ::: "memory"); }

// fma(x[n], x[n], acc) over n = 0 .. N - 1 in order from zero, x a
// 16-byte-aligned run in shared memory. DEEP: loads 16 steps ahead of the
// chain (two register buffers of four float4), for kernels with registers
// to spare; else four steps a load as the loop comes.
__device__ __forceinline__ void ld16f(const float* x, int b, float4 (&r)[4]) {
#pragma unroll
    for (int e = 0; e < 4; e++) r[e] = *(const float4*)(x + 16 * b + 4 * e);
}
__device__ __forceinline__ float sqfma16(const float4 (&r)[4], float acc) {
#pragma unroll
    for (int e = 0; e < 4; e++) {
        acc = __fmaf_rn(r[e].x, r[e].x, acc);
        acc = __fmaf_rn(r[e].y, r[e].y, acc);
        acc = __fmaf_rn(r[e].z, r[e].z, acc);
        acc = __fmaf_rn(r[e].w, r[e].w, acc);
    }
    return acc;
}
template <int N, bool DEEP>
__device__ __forceinline__ float sq_chain(const float* x) {
    static_assert(N % 32 == 0, "pairs of 16-step batches");
    float acc = 0.f;
    if (!DEEP) {
#pragma unroll 4
        for (int k4 = 0; k4 < N / 4; k4++) {
            const float4 t = *(const float4*)(x + 4 * k4);
            acc = __fmaf_rn(t.x, t.x, acc);
            acc = __fmaf_rn(t.y, t.y, acc);
            acc = __fmaf_rn(t.z, t.z, acc);
            acc = __fmaf_rn(t.w, t.w, acc);
        }
        return acc;
    }
    float4 a[4], b[4];
    ld16f(x, 0, a);
#pragma unroll 1
    for (int s = 0; s < N / 16; s += 2) {
        ld16f(x, s + 1, b);
        acc = sqfma16(a, acc);
        if (s + 2 < N / 16) ld16f(x, s + 2, a);
        acc = sqfma16(b, acc);
    }
    return acc;
}

// dot16_combine over lanes 0-15 of a warp (chain c in lane c); the total is
// valid in lane 0. Every lane of the warp must call it.
__device__ __forceinline__ float dot16_combine_warp(float acc, int ln) {
    const unsigned F = 0xffffffffu;
    const int l = ln & 3;
    float a4 = __shfl_sync(F, acc, 4 + l), a8 = __shfl_sync(F, acc, 8 + l), a12 = __shfl_sync(F, acc, 12 + l);
    float t = __fadd_rn(__fadd_rn(__fadd_rn(a8, a12), a4), acc);
    float t1 = __shfl_sync(F, t, 1), t2 = __shfl_sync(F, t, 2), t3 = __shfl_sync(F, t, 3);
    return __fadd_rn(__fadd_rn(t, t1), __fadd_rn(t2, t3));
}

// Four per-lane integer sums reduced across the warp: afterwards lanes
// 8i..8i+7 hold value i's total (i = (lane >> 3)'s bits 16, 8 as 2, 1).
__device__ __forceinline__ int reduce4_scatter(const int s[4], int ln) {
    const unsigned F = 0xffffffffu;
    int h[2];
    const bool u16 = ln & 16, u8 = ln & 8;
#pragma unroll
    for (int j = 0; j < 2; j++) h[j] = (u16 ? s[j + 2] : s[j]) + __shfl_xor_sync(F, u16 ? s[j] : s[j + 2], 16);
    int r = (u8 ? h[1] : h[0]) + __shfl_xor_sync(F, u8 ? h[0] : h[1], 8);
    r += __shfl_xor_sync(F, r, 4);
    r += __shfl_xor_sync(F, r, 2);
    r += __shfl_xor_sync(F, r, 1);
    return r;
}

// The mHC read's block barrier: PART when its MHC_THREADS threads are part
// of a wider CTA whose other threads may have left.
template <bool PART>
__device__ __forceinline__ void mhc_bar() {
    if (PART)
        asm volatile("bar.sync 2, %0;\n" ::"n"(MHC_THREADS) : "memory");
    else
        __syncthreads();
}

// infer.rs:1359-1426 for row m, by threads 0 .. MHC_THREADS - 1 of a CTA
// (MINB: the CTAs an SM its launch bounds allow). The lanes are normalized
// by one rms and quantized to int8 (no rotation) in registers; the 24 int8
// gate dots are per-thread dp4a partials over 16-byte runs of the gate
// rows, reduced exactly across the CTA. Then warp 5 stores the post block's
// gate projections for mhc_gates_kernel while warps
// 0-4 form u from the pre gates, apply the engram gate (when the layer has a
// site: ekv [M][1536] keys, evals [M][768]), the input ZC-RMSNorm and A8 of
// the normed row (act/sx for the q|k|v|gate matmul; x1o is the residual).
template <int MINB, bool PART = false>
__device__ __forceinline__ void mhc_read_row(const LayerW& w, int lane_own, const float* xs, float* u, float* p, const float* ekv,
                                             const float* evals, float* x1o, int8_t* act, float* sx, int m) {
    // dot16 operands loaded 16 at a time in the eight-CTA variant (42
    // registers), all 48 at once in the other
    constexpr int MHC_B16 = MINB == 1 ? 48 : 16;
    // the four streams chain-major: element e at (e % 16) * MHC_XS + e / 16,
    // so each of the sixteen chains of the rms dot reads 16-byte runs;
    // later the norm's scratch rows
    __shared__ __align__(16) float xt[16 * MHC_XS];
    __shared__ __align__(16) float x1[768];
    __shared__ __align__(16) float nin[768], ek[768], ev[768];
    __shared__ int red24[6][24];
    __shared__ float red[6];
    __shared__ float part[32];
    __shared__ float hp[4];
    __shared__ float sc_s[4];
    const int tid = threadIdx.x, warp = tid >> 5, ln = tid & 31;
    // the input norm's operands, fetched by the threads that will use them
    if (tid < MHC_NORM_THREADS) {
        for (int k = tid; k < 192; k += MHC_NORM_THREADS) {
            cp_async16(nin + 4 * k, w.norm_in + 4 * k, true);
            if (ekv) {
                cp_async16(ek + 4 * k, ekv + (size_t)m * 1536 + 4 * k, true);
                cp_async16(ev + 4 * k, evals + (size_t)m * 768 + 4 * k, true);
            }
        }
    }
    asm volatile("cp.async.commit_group;\n" ::);
    float v[16];
    {
        const float4* xr = (const float4*)(xs + (size_t)m * 3072) + 4 * tid;
#pragma unroll
        for (int i = 0; i < 4; i++) {
            float4 t = xr[i];
            v[4 * i] = t.x;
            v[4 * i + 1] = t.y;
            v[4 * i + 2] = t.z;
            v[4 * i + 3] = t.w;
        }
#pragma unroll
        for (int j = 0; j < 16; j++) xt[j * MHC_XS + tid] = v[j];  // element 16 tid + j
    }
    mhc_bar<PART>();
    if (warp == 0) {
        float acc = 0.f;
        if (ln < 16) acc = sq_chain<192, MINB == 1>(xt + ln * MHC_XS);
        float ss = dot16_combine_warp(acc, ln);
        if (ln == 0) sc_s[0] = rinv(ss, 3072);
    }
    mhc_bar<PART>();
    const float r = sc_s[0];
    float a = 0.f;
    {
#pragma unroll
        for (int k = 0; k < 16; k++) {
            v[k] = __fmul_rn(v[k], r);
            a = fmaxf(a, fabsf(v[k]));
        }
        a = warp_max(a);
        if (ln == 0) red[warp] = a;
    }
    mhc_bar<PART>();
    float mx = red[0];
#pragma unroll
    for (int k = 1; k < 6; k++) mx = fmaxf(mx, red[k]);
    const float sxv = mx > 0.f ? __fmul_rn(mx, ND_K127) : 1.0f;
    {
        const float inv = __fdiv_rn(1.0f, sxv);
        int wd[4];
#pragma unroll
        for (int i = 0; i < 4; i++) {
            uint32_t b0 = (uint8_t)q8_round(v[4 * i], inv), b1 = (uint8_t)q8_round(v[4 * i + 1], inv);
            uint32_t b2 = (uint8_t)q8_round(v[4 * i + 2], inv), b3 = (uint8_t)q8_round(v[4 * i + 3], inv);
            wd[i] = (int)(b0 | (b1 << 8) | (b2 << 16) | (b3 << 24));
        }
        // the 24 gate dots: thread t owns bytes 16 t .. 16 t + 15 of the row
        const int4* wq = (const int4*)w.phi_q + tid;
#pragma unroll
        for (int bt = 0; bt < 6; bt++) {
            int s4[4];
#pragma unroll
            for (int kk = 0; kk < 4; kk++) {
                const int4 g = __ldg(wq + (bt * 4 + kk) * 192);
                s4[kk] = __dp4a(g.w, wd[3], __dp4a(g.z, wd[2], __dp4a(g.y, wd[1], __dp4a(g.x, wd[0], 0))));
            }
            int tot = reduce4_scatter(s4, ln);
            if ((ln & 7) == 0) red24[warp][bt * 4 + ((ln & 16) ? 2 : 0) + ((ln & 8) ? 1 : 0)] = tot;
        }
    }
    mhc_bar<PART>();
    if (warp == 5) {
        // the post block's gate projections (pr[4..23]) into gates[m][4..23];
        // mhc_gates_kernel turns them into hpost and the Sinkhorn matrix
        if (ln < 20) {
            int tot = 0;
#pragma unroll
            for (int wp = 0; wp < 6; wp++) tot += red24[wp][4 + ln];
            p[(size_t)m * 24 + 4 + ln] = __fmul_rn(__fmul_rn(sxv, w.phi_s[4 + ln]), (float)tot);
        }
        return;
    }
    const int lt = tid;  // 0..159
    if (lt < 4) {
        int tot = 0;
#pragma unroll
        for (int wp = 0; wp < 6; wp++) tot += red24[wp][lt];
        float pr = __fmul_rn(__fmul_rn(sxv, w.phi_s[lt]), (float)tot);
        float off = lt == lane_own ? 4.0f : -4.0f;
        float z = __fadd_rn(__fadd_rn(__fmul_rn(pr, w.a_pre), off), w.b_pre[lt]);
        hp[lt] = __fdiv_rn(1.0f, __fadd_rn(lexpf(-z), 1.0f));
    }
    norm_bar();
    for (int ch = lt; ch < 768; ch += MHC_NORM_THREADS) {
        const float* xc = xt + (ch & 15) * MHC_XS + (ch >> 4);
        float o = __fmul_rn(xc[0], hp[0]);
        o = __fmaf_rn(xc[48], hp[1], o);
        o = __fmaf_rn(xc[96], hp[2], o);
        o = __fmaf_rn(xc[144], hp[3], o);
        u[(size_t)m * 768 + ch] = o;
        x1[ch] = o;
    }
    asm volatile("cp.async.wait_group 0;\n" ::);
    norm_bar();
    // infer.rs:1397-1426: the engram gate, the input norm, A8
    float* na = xt;
    float* nb = xt + 768;
    if (ekv) {
        if (lt < 16) part[lt] = dot16_sq<768, MHC_B16>(x1, lt);
        else if (lt < 32) part[lt] = dot16_sq<768, MHC_B16>(ek, lt - 16);
        norm_bar();
        if (lt == 0) sc_s[1] = rinv(dot16_combine(part), 768);
        if (lt == 1) sc_s[2] = rinv(dot16_combine(part + 16), 768);
        norm_bar();
        for (int k = lt; k < 768; k += MHC_NORM_THREADS) {
            na[k] = __fmul_rn(x1[k], sc_s[1]);
            nb[k] = __fmul_rn(ek[k], sc_s[2]);
        }
        norm_bar();
        if (lt < 16) part[lt] = dot16_chain<768, MHC_B16 / 2>(na, nb, lt);
        norm_bar();
        if (lt == 0) {
            float dab = dot16_combine(part);
            sc_s[3] = __fdiv_rn(1.0f, __fadd_rn(lexpf(__fdiv_rn(-dab, __fsqrt_rn(768.0f))), 1.0f));
        }
        norm_bar();
        const float alpha = sc_s[3];
        for (int k = lt; k < 768; k += MHC_NORM_THREADS) x1[k] = __fmaf_rn(ev[k], alpha, x1[k]);
        norm_bar();
    }
    if (warp == 0) {
        float acc = ln < 16 ? dot16_sq<768, MHC_B16>(x1, ln) : 0.f;
        float ss = dot16_combine_warp(acc, ln);
        if (ln == 0) sc_s[0] = rinv(ss, 768);
    }
    norm_bar();
    const float rn = sc_s[0];
    for (int k = lt; k < 768; k += MHC_NORM_THREADS) {
        x1o[(size_t)m * 768 + k] = x1[k];
        float t = __fmul_rn(x1[k], rn);
        na[k] = __fmaf_rn(t, nin[k], t);
    }
    norm_bar();
    for (int gw = warp; gw < 6; gw += 5) {
        float vv[4];
#pragma unroll
        for (int k = 0; k < 4; k++) vv[k] = na[gw * 128 + 4 * ln + k];
        prep_group_warp(vv, ln, act + ((size_t)m * 6 + gw) * 128, sx + (size_t)m * 6 + gw);
    }
}

template <int MINB>
__global__ void __launch_bounds__(MHC_THREADS, MINB) mhc_read_kernel(LayerW w, int lane_own, const float* xs, float* u, float* p,
                                                                  const float* ekv, const float* evals, float* x1o, int8_t* act,
                                                                  float* sx) {
    pdl_launch_dependents();
    pdl_wait();
    mhc_read_row<MINB>(w, lane_own, xs, u, p, ekv, evals, x1o, act, sx, blockIdx.x);
}

void launch_mhc_read(LayerW w, int lane, const float* xs, int M, float* u, float* p, const float* ekv, const float* evals,
                     float* x1, int8_t* act, float* sx, cudaStream_t st) {
    COUNT_LAUNCH();
    // eight CTAs an SM (42 registers a thread) keep a batch of up to 1184
    // rows in one wave; a batch of at most one row an SM takes the variant
    // with the registers to run its chains from registers
    if (M <= sm_count())
        launch_pdl(mhc_read_kernel<1>, dim3(M), dim3(MHC_THREADS), 0, st, w, lane, xs, u, p, ekv, evals, x1, act, sx);
    else
        launch_pdl(mhc_read_kernel<8>, dim3(M), dim3(MHC_THREADS), 0, st, w, lane, xs, u, p, ekv, evals, x1, act, sx);
}

// infer.rs:1580-1586 for one row per warp, from the projections the mHC read
// left in gates[m][4..23] (pr[4..7] for hpost, pr[8..23] for the residual
// mix): lanes 16-19 hpost, lanes 0-15 the 4x4 Sinkhorn (sinkhorn64,
// 2501-2525) in f64, one element each: the pairwise row and column sums are
// xor-shuffles, which add (e0 + e1) + (e2 + e3) as the reference does. The
// results replace the row's gates[0..19]: hpost[4], then hres[16].
__global__ void __launch_bounds__(256) mhc_gates_kernel(LayerW w, int lane_own, int M, float* p) {
    pdl_launch_dependents();
    pdl_wait();
    const int m = blockIdx.x * 8 + (threadIdx.x >> 5), ln = threadIdx.x & 31;
    if (m >= M) return;
    const unsigned F = 0xffffffffu;
    float* g = p + (size_t)m * 24;
    const float pk = ln < 20 ? g[4 + ln] : 0.f;
    const float pj = __shfl_sync(F, pk, ln & 3);
    const float pres = __shfl_sync(F, pk, (ln & 15) + 4);
    const int rr = (ln & 15) >> 2;
    float zr = ln < 16 ? __fmaf_rn(pres, w.a_res, w.b_res[ln & 15]) : 0.f;
    float zm = fmaxf(fmaxf(__shfl_sync(F, zr, rr * 4), __shfl_sync(F, zr, rr * 4 + 1)),
                     fmaxf(__shfl_sync(F, zr, rr * 4 + 2), __shfl_sync(F, zr, rr * 4 + 3)));
    double e = exp(__dsub_rn((double)zr, (double)zm));
    for (int it = 0; it < 20; it++) {
        // __drcp_rn is the correctly rounded 1.0 / x
        double s2 = __dadd_rn(e, __shfl_xor_sync(F, e, 1));
        double s4 = __dadd_rn(s2, __shfl_xor_sync(F, s2, 2));
        e = __dmul_rn(e, __drcp_rn(s4));
        double c2 = __dadd_rn(e, __shfl_xor_sync(F, e, 4));
        double c4 = __dadd_rn(c2, __shfl_xor_sync(F, c2, 8));
        e = __dmul_rn(e, __drcp_rn(c4));
    }
    __syncwarp();  // every lane has read its projection before any is replaced
    if (ln >= 16 && ln < 20) {
        const int j = ln - 16;
        float off = j == lane_own ? 0.0f : -4.0f;
        float z = __fadd_rn(__fadd_rn(__fmul_rn(pj, w.a_post), off), w.b_post[j]);
        g[j] = __fdiv_rn(2.0f, __fadd_rn(lexpf(-z), 1.0f));
    }
    if (ln < 16) g[4 + ln] = (float)e;
}

void launch_mhc_gates(LayerW w, int lane, int M, float* gates, cudaStream_t st) {
    COUNT_LAUNCH();
    launch_pdl(mhc_gates_kernel, dim3(cdiv(M, 8)), dim3(256), 0, st, w, lane, M, gates);
}

// ------------------------------------------------ conv taps, RoPE, int8 KV

// infer.rs:1430-1526 (chunk rows) as unit work (infer/step.rs:468-516): per
// row, 12 q heads, 2 k heads and 2 v heads, one unit each. A CTA takes a
// row: with UPW = 2, eight warps, warp w units w and w + 8, every load of
// both units issued before either is worked on (a row in 256 threads, so a
// large batch's rows are resident at once: 1024 rows fit 148 SMs x 8); with
// UPW = 1, sixteen warps, one unit each (the shorter chain for small
// batches). The taps read earlier rows of this chunk, else the pre-tap
// history, else zeros.
// Unit u of a row's pre-tap values: its first column in the q|k|v part of
// the projection, its taps' row stride and column, its width, its taps.
__device__ __forceinline__ void conv_unit_of(const LayerW& w, int unit, int& start, int& cw, int& cc, int& len, const float*& wt) {
    if (unit < 12) { start = unit * 48; cw = 576; cc = unit * 48; len = 48; wt = w.q_taps; }
    else if (unit < 14) { int kh = unit - 12; start = 576 + kh * 48; cw = 96; cc = kh * 48; len = 48; wt = w.k_taps; }
    else { int vh = unit - 14; start = 672 + vh * 64; cw = 128; cc = vh * 64; len = 64; wt = w.v_taps; }
}

// One (row, unit) of the conv by one warp, the lane's channels k = lane,
// lane + 32 (< the unit's width) given with their current pre-tap value
// and the two before (zero where no earlier row exists): the row's pre-tap
// values join the history ring (infer.rs:1486-1488; its slot is none of the
// two that rows 0 and 1 read), the taps run into x (64 floats of shared
// memory), then q and k heads take zcn and RoPE (qbuf for q), k and v heads
// int8 at this position's cache slot.
__device__ __forceinline__ void conv_unit(const LayerW& w, int l, int unit, const Caches& c, int s, int i, int pos, int m,
                                          size_t hrow0, const float (&cur)[2], const float (&prev)[2][2], float* x,
                                          const float* cosr, const float* sinr, float* qbuf, int lane) {
    int start, cw, cc, len;
    const float* wt;
    conv_unit_of(w, unit, start, cw, cc, len, wt);
#pragma unroll
    for (int t = 0; t < 2; t++) {
        const int k = lane + 32 * t;
        if (k < len) {
            c.hist[(hrow0 + pos % HIST_RING) * 800 + start + k] = cur[t];
            float o = __fmul_rn(wt[cc + k], cur[t]);
            o = __fmaf_rn(wt[cw + cc + k], prev[t][0], o);
            o = __fmaf_rn(wt[2 * cw + cc + k], prev[t][1], o);
            x[k] = o;
        }
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
        float rr = rinv(dot16_combine(chains), 48);
        const float* scale = unit < 12 ? w.q_norm : w.k_norm;
        float t0 = __fmul_rn(x[lane], rr);
        float y0 = __fmaf_rn(t0, scale[lane], t0);
        float y1 = 0.f;
        if (lane < 16) {
            float t1 = __fmul_rn(x[lane + 32], rr);
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
        int8_t* vg = c.v8 + ((((size_t)s * c.L + l) * 2 + vh) * c.vgroups + (pos >> 2)) * 256 + (pos & 3);
        for (int k = lane; k < 64; k += 32) vg[k * 4] = q8_round(x[k], inv);
        if (lane == 0) c.vs[row] = sc;
    }
}

template <int UPW>
__global__ void __launch_bounds__(512 / UPW, 8 / (3 - UPW)) conv_rope_kv_kernel(LayerW w, int l, const float* proj, Caches c,
                                                                             int T, const int32_t* p0p, int hist_base,
                                                                             const float* cosr, const float* sinr, float* qbuf) {
    constexpr int WARPS = 16 / UPW;
    pdl_launch_dependents();
    pdl_wait();
    const int p0 = *p0p;
    __shared__ float buf[16][64];
    const int m = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int s = T == 1 ? m : m / T, i = T == 1 ? 0 : m % T, pos = p0 + i;
    const size_t hrow0 = ((size_t)s * c.L + l) * HIST_RING;
    // every row load of the lane's (at most two) channels of the warp's
    // units first, then the tap weights (cache-resident), history writes
    // and taps
    float cur[UPW][2], prev[UPW][2][2];
#pragma unroll
    for (int r = 0; r < UPW; r++) {
        int start, cw, cc, len;
        const float* wt;
        conv_unit_of(w, warp + WARPS * r, start, cw, cc, len, wt);
#pragma unroll
        for (int t = 0; t < 2; t++) {
            const int k = lane + 32 * t;
            cur[r][t] = 0.f;
            prev[r][t][0] = prev[r][t][1] = 0.f;
            if (k < len) {
                cur[r][t] = proj[(size_t)m * 1568 + start + k];
#pragma unroll
                for (int j = 1; j < 3; j++) {
                    const int pj = pos - j;
                    if (i - j >= 0) prev[r][t][j - 1] = proj[(size_t)(m - j) * 1568 + start + k];
                    else if (pj >= hist_base && pj >= 0) prev[r][t][j - 1] = c.hist[(hrow0 + pj % HIST_RING) * 800 + start + k];
                }
            }
        }
    }
#pragma unroll
    for (int r = 0; r < UPW; r++)
        conv_unit(w, l, warp + WARPS * r, c, s, i, pos, m, hrow0, cur[r], prev[r], buf[warp + WARPS * r], cosr, sinr, qbuf, lane);
}

// The q|k|v|gate GEMV and the conv in one launch, for one-token steps of up
// to GEMV_MAXM rows (row m is sequence m): CTA u < 16 computes unit u's
// pre-tap rows of the projection (q heads 0-11: 48 rows, k heads: 48, v
// heads: 64; two rows a warp of 32), then warp m runs that unit's conv for
// row m; CTAs 16-27 compute the gate rows, 64 each. Every weight row's codes are read before
// the wait on the predecessor, as in the GEMV; the history rows (earlier
// steps') after it. Each value is computed as cq_gemv_kernel and
// conv_rope_kv_kernel compute it.
constexpr int QKVC_CTAS = 16 + 768 / 64, QKVC_WARPS = 32;
template <int FMT>
__global__ void __launch_bounds__(32 * QKVC_WARPS) qkvg_conv_kernel(DevMat W, const int8_t* act, const float* sx, int M, float* proj, LayerW w,
                                                        int l, Caches c, const int32_t* p0p, int hist_base, const float* cosr,
                                                        const float* sinr, float* qbuf) {
    pdl_launch_dependents();
    __shared__ float buf[GEMV_MAXM][64];
    const int u = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int r0, nr;
    if (u < 12) r0 = 48 * u, nr = 48;
    else if (u < 14) r0 = 576 + 48 * (u - 12), nr = 48;
    else if (u < 16) r0 = 672 + 64 * (u - 14), nr = 64;
    else r0 = 800 + 64 * (u - 16), nr = 64;
    // two weight rows a warp (a unit has at most 64)
    GemvRow rr[2];
#pragma unroll
    for (int k = 0; k < 2; k++)
        if (warp + QKVC_WARPS * k < nr) gemv_row_load<FMT>(W, r0 + warp + QKVC_WARPS * k, lane, rr[k]);
    pdl_wait();
    // the conv warps (warp m of a unit CTA) request their history rows
    // first, so the loads run under the GEMV
    const bool conv_warp = u < 16 && warp < M;
    const int m = warp, pos = *p0p;
    const size_t hrow0 = ((size_t)m * c.L + l) * HIST_RING;
    int start = 0, cw, cc, len = 0;
    const float* wt;
    if (u < 16) conv_unit_of(w, u, start, cw, cc, len, wt);
    float cur[2], prev[2][2];
#pragma unroll
    for (int t = 0; t < 2; t++) {
        const int k = lane + 32 * t;
        cur[t] = 0.f;
        prev[t][0] = prev[t][1] = 0.f;
        if (conv_warp && k < len)
#pragma unroll
            for (int j = 1; j < 3; j++) {
                const int pj = pos - j;
                if (pj >= hist_base && pj >= 0) prev[t][j - 1] = c.hist[(hrow0 + pj % HIST_RING) * 800 + start + k];
            }
    }
#pragma unroll
    for (int k = 0; k < 2; k++)
        if (warp + QKVC_WARPS * k < nr) gemv_row_out<FMT>(W, rr[k], r0 + warp + QKVC_WARPS * k, lane, act, sx, M, proj, 1568, 0);
    if (u >= 16) return;
    __syncthreads();  // the unit's pre-tap rows are in proj
    if (!conv_warp) return;
#pragma unroll
    for (int t = 0; t < 2; t++) {
        const int k = lane + 32 * t;
        if (k < len) cur[t] = proj[(size_t)m * 1568 + start + k];
    }
    conv_unit(w, l, u, c, m, 0, pos, m, hrow0, cur, prev, buf[m], cosr, sinr, qbuf, lane);
}

cudaError_t launch_qkvg_conv(DevMat W, const int8_t* act, const float* sx, int M, float* proj, LayerW w, int l, Caches c,
                             int hist_base, const float* cosr, const float* sinr, float* qbuf, cudaStream_t st) {
    static_assert(QKVG_CONV_MAX_ROWS <= GEMV_MAXM, "the GEMV's rows");
    if (!W.w8 || W.groups != 6 || W.in_dim != 768 || W.out != 1568 || M < 1 || M > QKVG_CONV_MAX_ROWS ||
        (W.width != 2 && W.width != 3 && W.width != 4))
        return cudaErrorInvalidValue;
    COUNT_LAUNCH();
    if (W.width == 4)
        launch_pdl(qkvg_conv_kernel<4>, dim3(QKVC_CTAS), dim3(32 * QKVC_WARPS), 0, st, W, act, sx, M, proj, w, l, c, c.len, hist_base, cosr, sinr, qbuf);
    else if (W.width == 2)
        launch_pdl(qkvg_conv_kernel<2>, dim3(QKVC_CTAS), dim3(32 * QKVC_WARPS), 0, st, W, act, sx, M, proj, w, l, c, c.len, hist_base, cosr, sinr, qbuf);
    else
        launch_pdl(qkvg_conv_kernel<8>, dim3(QKVC_CTAS), dim3(32 * QKVC_WARPS), 0, st, W, act, sx, M, proj, w, l, c, c.len, hist_base, cosr, sinr, qbuf);
    return cudaSuccess;
}

void launch_conv_rope_kv(LayerW w, int l, const float* proj, Caches c, int S, int T, int p0, int hist_base, const float* cosr,
                         const float* sinr, float* qbuf, cudaStream_t st) {
    COUNT_LAUNCH();
    // 512-thread CTAs at 32 registers fit four an SM: one wave up to 592 rows
    if (S * T <= 592)
        launch_pdl(conv_rope_kv_kernel<1>, dim3(S * T), dim3(512), 0, st, w, l, proj, c, T, c.len, hist_base, cosr, sinr, qbuf);
    else
        launch_pdl(conv_rope_kv_kernel<2>, dim3(S * T), dim3(256), 0, st, w, l, proj, c, T, c.len, hist_base, cosr, sinr, qbuf);
}

// ------------------------------------------------------------- attention

// attend_head_ref (infer.rs:1871-2004) for one (row, head): int8 query,
// the engine's key chunks (key_chunks, 2093-2101), scores with the 4-block
// order rule, chunk_exp (2222-2318), 21-bit digits (2171-2217), integer P.V,
// and the merge (2143-2166); then the gate (1548-1552).
constexpr int ATT_MAXCHUNK = 256, ATT_MAXPARTS = ATT_MAX_KEYS / ATT_MAXCHUNK;

// a / b for 0 <= a < 2^24 and 0 < b: a float quotient, then one step of
// correction each way, exact (the integer divide's generic sequence is
// several times longer, and every warp of the attention kernel runs these)
__device__ __forceinline__ int small_div(int a, int b) {
    int q = (int)__fdividef((float)a, (float)b);
    if ((q + 1) * b <= a) q++;
    if (q * b > a) q--;
    return q;
}

__device__ __forceinline__ void key_chunks_dev(int n, bool nested, int* count, int* chunk) {
    int k = nested ? 1 : 4;  // (2 * NATIVE_TEAM / nkv).max(1), NATIVE_TEAM = 4, nkv = 2
    int c = (n + 255) / 256;
    if (k * 64 <= n && c < k) c = k;
    int cm = c > 1 ? c : 1;
    int ch = (small_div(n + cm - 1, cm) + 15) / 16 * 16;
    *chunk = ch;
    *count = ch > 0 ? small_div(n + ch - 1, ch) : 0;
}

// One CTA per (row, kv head) serves the kv head's 6 query heads: the chunk's
// key rows and value groups (the cache keeps values as words of four
// positions' bytes per dimension, positions 4g..4g+3, which the digit dot
// products take as they are) are copied once into shared memory with
// cp.async, issued before the queries are quantized; then warp h runs head
// h through scores, max, numerators, the fixed-order sum, digits, P.V,
// merge and gate with no block-wide barrier. Digits sit at the chunk's
// offset within its first group, zero outside the chunk. P.V is an int8
// matrix product on the tensor cores (mma.sync m16n8k32, exact int32 sums,
// so the result is the reference's integer dot whatever the order): A =
// the value bytes of 16 dimensions by 32 keys (8 groups), which the cache's
// group words already hold in the fragment's 4-keys-per-register order,
// B = the same keys' three digit planes. A key's score, numerator and
// weight stay in the registers of the lane that owns it until the weights
// go to shared memory for the digits. Rows with more than one chunk keep per-chunk
// parts in dynamic shared memory sized for the longest key list of the
// launch; a one-chunk row keeps its part in registers, so a launch of
// one-chunk rows needs no parts space.
// A chunk spans at most ATT_MAXCHUNK / 4 + 3 value groups (a group cut at
// each end of the sink run and of the ring run); the P.V loop reads whole
// steps of 8 groups, so the buffers hold a multiple of 8.
constexpr int ATT_HEADS = 6, ATT_THREADS = ATT_HEADS * 32, ATT_MAXGROUPS = (ATT_MAXCHUNK / 4 + 3 + 7) / 8 * 8;
static_assert(ATT_MAXGROUPS % 8 == 0 && ATT_MAXGROUPS >= ATT_MAXCHUNK / 4 + 3, "whole 8-group steps");
struct AttSmem {
    int8_t k[ATT_MAXCHUNK][48];
    // value group w: the words of dimensions 0..63, the 16-byte run of
    // dimensions 4c..4c+3 at word (4c) ^ (8 (w & 3)), so the P.V fragment
    // loads of four consecutive groups fall in four distinct bank octets
    int vg[ATT_MAXGROUPS][64];
    float ks[ATT_MAXCHUNK], vs[ATT_MAXCHUNK];
    // per head: the P.V plane sums on their way to the lanes that own
    // them (3 x 72 words), at the end the gated outputs (6 x 64 in all)
    float s[ATT_HEADS][ATT_MAXCHUNK];
    // digit plane (hi, mid, lo) of value group g: one word, the four
    // positions 4g..4g+3 in its bytes
    int dig[ATT_HEADS][3][ATT_MAXGROUPS];
    __align__(16) int8_t q8[ATT_HEADS][48];
    // followed, when a row of the launch has more than one chunk, by parts:
    // [ATT_HEADS][count][66] floats (m, sum, o[64])
};
static_assert(3 * 72 <= ATT_MAXCHUNK, "the P.V scratch fits a score row");

// Numerators a lane holds: key k = lane + 32 i in slot i.
constexpr int ATT_KPL = ATT_MAXCHUNK / 32;
// Key k's value from the lane that holds it; every lane of the warp calls
// it, with keys of one slot (k / 32 the same in every lane).
__device__ __forceinline__ float att_key_val(const float (&ev)[ATT_KPL], int k) {
    const int slot = k >> 5;
    float v = 0.f;
#pragma unroll
    for (int i = 0; i < ATT_KPL; i++)
        if (i == slot) v = ev[i];
    return __shfl_sync(0xffffffffu, v, k & 31);
}

__device__ __forceinline__ void mma_s8_acc(int (&d)[4], const uint32_t (&a)[4], const uint32_t (&b)[2]) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

template <int MINB>
__global__ void __launch_bounds__(ATT_THREADS, MINB) attention_kernel(const float* qbuf, const float* proj, Caches c, int l, int T,
                                                                const int32_t* p0p, int window, int sink, int ring, float* att,
                                                                int8_t* act, float* sx) {
    pdl_launch_dependents();
    pdl_wait();
    const int p0 = *p0p;
    extern __shared__ __align__(16) int8_t att_raw[];
    AttSmem& sm = *reinterpret_cast<AttSmem*>(att_raw);
    const int m = blockIdx.x, kvh = blockIdx.y, tid = threadIdx.x, lane = tid & 31, h = tid >> 5;
    const int s = T == 1 ? m : m / T, i = T == 1 ? 0 : m % T, pos = p0 + i;
    const bool nested = T > 1;
    // infer.rs:1781-1825 (key_ranges): the keys as runs of positions, A =
    // [aS, aE) then B = [bS, bE). Without an attention span A is the layer's
    // band; with one, A is the sink within the band and B the ring as of
    // the chunk's end (not cut by the band, as the engine has it). The cache
    // keeps every position, so no key of these runs has lost its slot.
    const int lo = window > 0 ? max(0, pos + 1 - window) : 0;
    int aE = pos + 1, bS = 0, bE = 0;
    if (ring > 0) {
        aE = max(lo, min(sink, pos + 1));
        bS = min(max(max(0, p0 + T - ring), sink), pos + 1);
        bE = pos + 1;
    }
    const int lenA = aE - lo, n = lenA + (bE - bS);
    // a chunk's keys [c0, c0 + len) as a segment of A (positions pA ..,
    // nA keys) then one of B (positions pB .., nB keys), with the value
    // groups each spans
    struct Seg {
        int nA, pA, gA0, ngA, nB, pB, gB0, ngB;
    };
    auto seg = [&](int c0, int len) {
        Seg g;
        g.nA = max(0, min(c0 + len, lenA) - c0);
        g.pA = lo + c0;
        g.gA0 = g.pA >> 2;
        g.ngA = g.nA > 0 ? ((g.pA + g.nA - 1) >> 2) - g.gA0 + 1 : 0;
        g.nB = len - g.nA;
        g.pB = bS + max(c0, lenA) - lenA;
        g.gB0 = g.pB >> 2;
        g.ngB = g.nB > 0 ? ((g.pB + g.nB - 1) >> 2) - g.gB0 + 1 : 0;
        return g;
    };
    int count, chunk;
    key_chunks_dev(n, nested, &count, &chunk);
    float* parts = reinterpret_cast<float*>(att_raw + ((sizeof(AttSmem) + 15) & ~(size_t)15)) + (size_t)h * count * 66;
    const int hh = kvh * ATT_HEADS + h;
    const size_t kvrow = (((size_t)s * c.L + l) * 2 + kvh) * c.cap;
    const int8_t* k8 = c.k8 + kvrow * 48;
    const int8_t* v8 = c.v8 + (((size_t)s * c.L + l) * 2 + kvh) * c.vgroups * 256;
    // the copies of chunk ci in two groups: key rows (each run of positions
    // one contiguous range of 48-byte rows) and scales, then the value
    // groups (A's, then B's), which P.V waits for
    auto issue_chunk = [&](int ci) {
        const int c0 = ci * chunk, len = min(chunk, n - c0);
        const Seg g = seg(c0, len);
        for (int idx = tid; idx < len * 3; idx += ATT_THREADS) {
            const int8_t* src = idx < 3 * g.nA ? k8 + (size_t)g.pA * 48 + idx * 16 : k8 + (size_t)g.pB * 48 + (idx - 3 * g.nA) * 16;
            cp_async16(&sm.k[0][0] + idx * 16, src, true);
        }
        for (int k = tid; k < len; k += ATT_THREADS) {
            const int p = k < g.nA ? g.pA + k : g.pB + k - g.nA;
            cp_async4(&sm.ks[k], c.ks + kvrow + p);
            cp_async4(&sm.vs[k], c.vs + kvrow + p);
        }
        asm volatile("cp.async.commit_group;\n" ::);
        for (int idx = tid; idx < (g.ngA + g.ngB) * 16; idx += ATT_THREADS) {
            const int w = idx >> 4, part = idx & 15, src = w < g.ngA ? g.gA0 + w : g.gB0 + w - g.ngA;
            cp_async16(&sm.vg[w][(part * 4) ^ ((w & 3) << 3)], v8 + (size_t)src * 256 + part * 16, true);
        }
        asm volatile("cp.async.commit_group;\n" ::);
    };
    // this head's query and gate rows are loaded before the chunk's copies
    // are issued, so their latency runs under the copies' issue
    const float* g = proj + (size_t)m * 1568 + 800 + hh * 64;
    const float2 gv = *(const float2*)(g + 2 * lane);  // this lane's two dimensions
    const float g0v = gv.x, g1v = gv.y;
    const float* qrow = qbuf + (size_t)m * 576 + hh * 48;
    const float x0 = qrow[lane], x1 = lane < 16 ? qrow[32 + lane] : 0.f;
    issue_chunk(0);
    float qs;
    {
        // quant_i8 of this head's query, scale folded with 1/sqrt(48) (infer.rs:1885)
        float a = warp_max(fmaxf(fabsf(x0), fabsf(x1)));
        float sc = a > 0.f ? __fmul_rn(a, ND_K127) : 1.0f;
        float inv = __fdiv_rn(1.0f, sc);
        sm.q8[h][lane] = q8_round(x0, inv);
        if (lane < 16) sm.q8[h][32 + lane] = q8_round(x1, inv);
        qs = __fmul_rn(sc, ND_INV_SQRT_QK);
    }
    float* srow = sm.s[h];
    float one0 = 0.f, one1 = 0.f, one_sum = 1.f;  // a one-chunk row's part
    for (int ci = 0; ci < count; ci++) {
        const int c0 = ci * chunk, len = min(chunk, n - c0), blocked = len / 4 * 4;
        const Seg sg = seg(c0, len);
        const int ng = sg.ngA + sg.ngB;
        asm volatile("cp.async.wait_group 1;\n" ::);  // keys and scales
        __syncthreads();
        // scores: (ks * dot) * qs in whole 4-blocks, (ks * qs) * dot after
        int qr[12];
#pragma unroll
        for (int e = 0; e < 3; e++) {
            const int4 v = ((const int4*)sm.q8[h])[e];
            qr[4 * e] = v.x;
            qr[4 * e + 1] = v.y;
            qr[4 * e + 2] = v.z;
            qr[4 * e + 3] = v.w;
        }
        // this lane's keys k = lane + 32 i stay in registers (ev[i]) from
        // the scores through the numerators, their sum and the weights
        float ev[ATT_KPL];
        float mx = -INFINITY;
#pragma unroll
        for (int i = 0; i < ATT_KPL; i++) {
            const int k = lane + 32 * i;
            ev[i] = 0.f;
            if (k < len) {
                const int4* kr = (const int4*)sm.k[k];
                int dot = 0;
#pragma unroll
                for (int e = 0; e < 3; e++) {
                    const int4 kv = kr[e];
                    dot = __dp4a(qr[4 * e], kv.x, dot);
                    dot = __dp4a(qr[4 * e + 1], kv.y, dot);
                    dot = __dp4a(qr[4 * e + 2], kv.z, dot);
                    dot = __dp4a(qr[4 * e + 3], kv.w, dot);
                }
                float ksv = sm.ks[k];
                float sv = k < blocked ? __fmul_rn(__fmul_rn(ksv, (float)dot), qs) : __fmul_rn(__fmul_rn(ksv, qs), (float)dot);
                ev[i] = sv;
                mx = fmaxf(mx, sv);
            }
        }
        mx = warp_max(mx);
        // numerators: the inline exp on whole 4-blocks, libm exp for the rest
#pragma unroll
        for (int i = 0; i < ATT_KPL; i++) {
            const int k = lane + 32 * i;
            if (k < len) {
                float dlt = __fsub_rn(ev[i], mx);
                ev[i] = k < blocked ? nexp(dlt) : lexpf(dlt);
            }
        }
        // chunk_exp's sum order (infer.rs:2279-2317): chain j < 4 adds the
        // first halves of the 8-blocks then the trailing 4-block, chain
        // j >= 4 the second halves; t_k = a_k + b_k; ((t0 + t1) + (t2 + t3)),
        // then the last 1-3 numerators one at a time. Chain j (lane j < 8)
        // takes block q's element q + j from lane (q + j) % 32, slot q / 32.
        const int n8 = len / 8 * 8;
        float a = 0.f;
#pragma unroll
        for (int i = 0; i < ATT_KPL; i++) {
            if (32 * i >= n8) break;
            const float y1 = __shfl_down_sync(0xffffffffu, ev[i], 8), y2 = __shfl_down_sync(0xffffffffu, ev[i], 16),
                        y3 = __shfl_down_sync(0xffffffffu, ev[i], 24);
            a = __fadd_rn(a, ev[i]);
            if (32 * i + 8 < n8) a = __fadd_rn(a, y1);
            if (32 * i + 16 < n8) a = __fadd_rn(a, y2);
            if (32 * i + 24 < n8) a = __fadd_rn(a, y3);
        }
        {
            const float yt = att_key_val(ev, n8 + (lane & 3));
            if (lane < 4 && blocked > n8) a = __fadd_rn(a, yt);
        }
        float tk = __fadd_rn(a, __shfl_down_sync(0xffffffffu, a, 4));  // lanes 0-3: a_k + b_k
        float t1 = __shfl_sync(0xffffffffu, tk, 1), t2 = __shfl_sync(0xffffffffu, tk, 2), t3 = __shfl_sync(0xffffffffu, tk, 3);
        float sum = __fadd_rn(__fadd_rn(tk, t1), __fadd_rn(t2, t3));
        {
            int ii = blocked;
            if (len - ii >= 2) {
                const float r0 = att_key_val(ev, ii), r1 = att_key_val(ev, ii + 1);
                sum = __fadd_rn(__fadd_rn(r0, sum), r1);
                ii += 2;
            }
            if (len - ii == 1) sum = __fadd_rn(sum, att_key_val(ev, ii));
        }
        sum = __shfl_sync(0xffffffffu, sum, 0);
        // weights times the value scales (in the registers), their max from zero
        float wm = 0.f;
#pragma unroll
        for (int i = 0; i < ATT_KPL; i++) {
            const int k = lane + 32 * i;
            if (k < len) {
                ev[i] = __fmul_rn(ev[i], sm.vs[k]);
                wm = fmaxf(wm, ev[i]);
            }
        }
        wm = warp_max(wm);
        const float qw = __fdiv_rn(ND_Q21, wm);
        // 21-bit digits: the chunk's group words start zero, then each lane
        // writes its keys' three digit bytes at the key's byte of the group
        // words (A's keys from byte pA % 4 on, B's after A's groups from
        // byte pB % 4 on); bytes of positions outside the chunk stay zero
        for (int g = lane; g < ng; g += 32) sm.dig[h][0][g] = sm.dig[h][1][g] = sm.dig[h][2][g] = 0;
        __syncwarp();
        {
            const int offA = sg.pA & 3, offB = 4 * sg.ngA + (sg.pB & 3) - sg.nA;
            int8_t* dg0 = (int8_t*)sm.dig[h][0];
#pragma unroll
            for (int i = 0; i < ATT_KPL; i++) {
                const int k = lane + 32 * i;
                if (k < len) {
                    const int kk = k < sg.nA ? k + offA : k + offB;
                    const int wq = (int)roundf(__fmul_rn(ev[i], qw));
                    dg0[kk] = (int8_t)(wq >> 14);
                    dg0[4 * ATT_MAXGROUPS + kk] = (int8_t)((wq >> 7) & 127);
                    dg0[8 * ATT_MAXGROUPS + kk] = (int8_t)(wq & 127);
                }
            }
        }
        asm volatile("cp.async.wait_group 0;\n" ::);  // value groups
        __syncthreads();
        // P.V on the tensor cores, 8 groups (32 keys) a step, as D = V x P:
        // A (16 x 32) is value dimensions 16 t .. 16 t + 15 by the step's
        // keys, which the cache's group words already hold four keys a
        // register (lane gid, tig: dimensions 16 t + gid, + 8 of groups
        // g0 = 8 ks + tig and g0 + 4); B (32 x 8) is the keys by the digit
        // planes, columns 0-2 (lane gid < 3 loads plane gid's words of g0
        // and g0 + 4, zero past the chunk's groups), the other columns zero.
        // Four m tiles cover the 64 dimensions; every sum is exact int32.
        {
            const int gid = lane >> 2, tig = lane & 3, steps = (ng + 7) >> 3, swz = tig << 3;
            const int* dp = sm.dig[h][gid < 3 ? gid : 0];
            int acc[4][4];
#pragma unroll
            for (int t = 0; t < 4; t++) acc[t][0] = acc[t][1] = acc[t][2] = acc[t][3] = 0;
            for (int ks = 0; ks < steps; ks++) {
                const int g0 = 8 * ks + tig, g1 = g0 + 4;
                const uint32_t b[2] = {gid < 3 && g0 < ng ? (uint32_t)dp[g0] : 0u, gid < 3 && g1 < ng ? (uint32_t)dp[g1] : 0u};
                const int* v0 = sm.vg[g0];
                const int* v1 = sm.vg[g1];
#pragma unroll
                for (int t = 0; t < 4; t++) {
                    const int d0 = (16 * t + gid) ^ swz, d1 = (16 * t + gid + 8) ^ swz;
                    const uint32_t a[4] = {(uint32_t)v0[d0], (uint32_t)v0[d1], (uint32_t)v1[d0], (uint32_t)v1[d1]};
                    mma_s8_acc(acc[t], a, b);
                }
            }
            // plane p's sums of dimension d go through the head's scratch row
            // to the lanes that own them: D (d, p) is lane (d % 8,
            // p / 2), element p % 2 (+ 2 for d % 16 >= 8)
            int* scr = reinterpret_cast<int*>(srow);
#pragma unroll
            for (int t = 0; t < 4; t++) {
                const int da = 16 * t + gid, db = da + 8;
                if (tig == 0) {
                    scr[da] = acc[t][0];
                    scr[72 + da] = acc[t][1];
                    scr[db] = acc[t][2];
                    scr[72 + db] = acc[t][3];
                } else if (tig == 1) {
                    scr[144 + da] = acc[t][0];
                    scr[144 + db] = acc[t][2];
                }
            }
            __syncwarp();
        }
        const int* scr = reinterpret_cast<const int*>(srow);
        const int2 dh = *(const int2*)&scr[2 * lane], dm = *(const int2*)&scr[72 + 2 * lane],
                   dl = *(const int2*)&scr[144 + 2 * lane];
        const float cw = __fmul_rn(wm, ND_C21);
        const float pv0 = __fmul_rn(__fmaf_rn(16384.f, (float)dh.x, __fmaf_rn(128.f, (float)dm.x, (float)dl.x)), cw);
        const float pv1 = __fmul_rn(__fmaf_rn(16384.f, (float)dh.y, __fmaf_rn(128.f, (float)dm.y, (float)dl.y)), cw);
        if (count == 1) {
            one0 = pv0;
            one1 = pv1;
            one_sum = sum;
        } else {
            float* pr = parts + ci * 66;
            pr[2 + 2 * lane] = pv0;
            pr[3 + 2 * lane] = pv1;
            if (lane == 0) {
                pr[0] = mx;
                pr[1] = sum;
            }
        }
        if (ci + 1 < count) {
            __syncthreads();  // every warp is done with this chunk's copies
            issue_chunk(ci + 1);
        }
    }
    __syncwarp();
    // merge_parts (infer.rs:2143-2166), then the gate (1548-1552)
    float out0, out1;
    if (count == 1) {
        float inv = __fdiv_rn(1.0f, one_sum);
        out0 = __fmul_rn(one0, inv);
        out1 = __fmul_rn(one1, inv);
    } else {
        float big = -1e30f;
        for (int ci = 0; ci < count; ci++) big = fmaxf(big, parts[ci * 66]);
        float a0 = 0.f, a1 = 0.f, total = 0.f;
        for (int ci = 0; ci < count; ci++) {
            const float* pr = parts + ci * 66;
            float wv = lexpf(__fsub_rn(pr[0], big));
            a0 = __fmaf_rn(pr[2 + 2 * lane], wv, a0);
            a1 = __fmaf_rn(pr[3 + 2 * lane], wv, a1);
            total = __fmaf_rn(wv, pr[1], total);
        }
        float inv = __fdiv_rn(1.0f, total);
        out0 = __fmul_rn(a0, inv);
        out1 = __fmul_rn(a1, inv);
    }
    float* o = att + (size_t)m * 768 + hh * 64;
    float y0 = __fdiv_rn(out0, __fadd_rn(nexp(-g0v), 1.0f));
    float y1 = __fdiv_rn(out1, __fadd_rn(nexp(-g1v), 1.0f));
    *(float2*)(o + 2 * lane) = make_float2(y0, y1);
    // A8 of the out projection's input (infer.rs:1556): this CTA's six heads
    // are exactly the 128-wide groups 3 kvh .. 3 kvh + 2.
    __syncthreads();
    float* gated = sm.s[0];  // [6][64] gated outputs, head-major
    gated[h * 64 + 2 * lane] = y0;
    gated[h * 64 + 2 * lane + 1] = y1;
    __syncthreads();
    if (h < 3) {
        float v[4];
#pragma unroll
        for (int k = 0; k < 4; k++) v[k] = gated[h * 128 + 4 * lane + k];
        const int grp = 3 * kvh + h;
        prep_group_warp(v, lane, act + ((size_t)m * 6 + grp) * 128, sx + (size_t)m * 6 + grp);
    }
}

extern const size_t ATT_SMEM_BASE = (sizeof(AttSmem) + 15) & ~(size_t)15;
extern const size_t ATT_SMEM = ATT_SMEM_BASE + (size_t)ATT_HEADS * ATT_MAXPARTS * 66 * 4;

void launch_attention(const float* qbuf, const float* proj, Caches c, int l, int S, int T, int p0, int window, int sink,
                      int ring, float* att, int8_t* act, float* sx, cudaStream_t st) {
    COUNT_LAUNCH();
    // key_chunks gives at most c = max(ceil(n / 256), k if n >= 64 k) chunks,
    // and the launch's longest key list is its last row's
    // sized for the batch's capacity, so a captured step stays valid at
    // every later position
    int nmax = c.cap;
    if (window > 0 && window < nmax && ring == 0) nmax = window;
    int most = std::max(1, (nmax + 255) / 256);
    if (T == 1 && nmax >= 256) most = std::max(most, 4);
    most = std::min(most, ATT_MAXPARTS);
    size_t smem = ATT_SMEM_BASE + (most > 1 ? (size_t)ATT_HEADS * most * 66 * 4 : 0);
    // five CTAs an SM (64 registers a thread) for batches; a launch of at
    // most one CTA an SM takes the variant with registers to spare
    if (2 * S * T <= sm_count())
        launch_pdl(attention_kernel<1>, dim3(dim3(S * T, 2)), dim3(ATT_THREADS), smem, st, qbuf, proj, c, l, T, c.len, window, sink,
                   ring, att, act, sx);
    else
        launch_pdl(attention_kernel<5>, dim3(dim3(S * T, 2)), dim3(ATT_THREADS), smem, st, qbuf, proj, c, l, T, c.len, window, sink,
                   ring, att, act, sx);
}

// ------------------------------------------------------------ post block


// infer.rs:1564-1606 with mlp_native (1610-1634), cond_weights (1640-1694),
// perm_fma (689-713), silu (2463-2496) and kron_native / mix8 (2322-2460).
// POST_ROWS rows per CTA of 64 POST_ROWS threads (a conditioning warp and a
// Kronecker warp a row), one CTA per SM: seven rows for a batch of 1024 (147
// of the 148 SMs; eight rows a CTA left 20 idle), four or two for batches
// that would leave SMs idle at seven (512 rows: 128 CTAs of four, not 74 of
// seven; each CTA's time shrinks with its rows). The layer's small
// weights (Kronecker factors, conditioning, diagonals, norms, permutations)
// are staged once into shared memory with cp.async, so every phase reads
// shared memory only (but the mHC write's inputs). A row's 1024-wide
// vectors use a padded layout (element p at (p / 32) * 36 + p % 32) and
// ping-pong between two buffers. The weights are requested before the
// predecessor kernel has finished, the rows' o, x1 and gates right after;
// u and the old streams are read by the mHC write itself, a round ahead
// (staging u in shared memory stalled its copies' issue for 1.9 K cycles).
// The post and residual gates (hpost, Sinkhorn) were computed by the mHC
// read.
constexpr int PV = 32 * 36 + 8;
template <int POST_ROWS>
struct PostSmem {
    float kf[6][1024];
    __align__(16) float cond_v[32 * COND_LD];
    float cond_u[8 * 1024];
    float d1[768], d2[1024], b2[1024], d3[1024], d4[768];
    float post_norm[768], pre_hada[768];
    int perm1[1024], perm2[1024];
    // the rows' buffers take 16-byte copies and loads at any row count
    __align__(16) float x2[POST_ROWS][768];
    __align__(16) float hs[POST_ROWS][4 * COND_LD];  // h2 = zcn(x2, pre_hada) chain-major, the conditioning input
    __align__(16) float buf[2][POST_ROWS][PV];
    __align__(16) float gates[POST_ROWS][24];
    float part[POST_ROWS][32];
    float sc[POST_ROWS][2];
    float wk[POST_ROWS][8];
};

static_assert(sizeof(PostSmem<7>) <= 232448, "seven rows fit one CTA's 227 KB of shared memory");

__device__ __forceinline__ int pv_idx(int p) { return (p >> 5) * 36 + (p & 31); }

template <int NT>
__device__ __forceinline__ void stage(void* dst, const void* src, int bytes, int tid) {
    for (int o = tid * 16; o < bytes; o += NT * 16) cp_async16((char*)dst + o, (const char*)src + o, true);
}

// The Kronecker passes: 32 threads (one warp) per CTA row, each a 4 x 8
// tile of outputs (rows r0..r0+3, columns c0..c0+7), so that one j step is
// three 16-byte shared loads for 16 paired fmas. Every output is one fma
// chain over j = 0..31 from zero, as kron_native (infer.rs:2442-2459) adds
// it. Row buffers are PV = 1160 floats apart.
// Pass 1: mt[c][r] = sum_j A[j][r] z[j][c] (A^T Z, stored transposed).
__device__ __forceinline__ void kron_pass1(const float* A, const float* z, float* mt, int r0, int c0) {
    float2 o[4][4];
#pragma unroll
    for (int a = 0; a < 4; a++)
#pragma unroll
        for (int b = 0; b < 4; b++) o[a][b] = make_float2(0.f, 0.f);
#pragma unroll 4
    for (int j = 0; j < 32; j++) {
        const float4 a0 = *(const float4*)(A + j * 32 + r0);
        const float4 z0 = *(const float4*)(z + j * 36 + c0), z1 = *(const float4*)(z + j * 36 + c0 + 4);
        const float ar[4] = {a0.x, a0.y, a0.z, a0.w};
        const float2 zp[4] = {make_float2(z0.x, z0.y), make_float2(z0.z, z0.w), make_float2(z1.x, z1.y), make_float2(z1.z, z1.w)};
#pragma unroll
        for (int a = 0; a < 4; a++)
#pragma unroll
            for (int b = 0; b < 4; b++) o[a][b] = fma2(make_float2(ar[a], ar[a]), zp[b], o[a][b]);
    }
#pragma unroll
    for (int b = 0; b < 8; b++) {
        const int bp = b >> 1;
        *(float4*)(mt + (c0 + b) * 36 + r0) = (b & 1) ? make_float4(o[0][bp].y, o[1][bp].y, o[2][bp].y, o[3][bp].y)
                                                      : make_float4(o[0][bp].x, o[1][bp].x, o[2][bp].x, o[3][bp].x);
    }
}

// Pass 2: t[r][c] = sum_j mt[j][r] B[j][c] ((A^T Z) B).
__device__ __forceinline__ void kron_pass2(const float* mt, const float* B, float* t, int r0, int c0) {
    float2 o[4][4];
#pragma unroll
    for (int a = 0; a < 4; a++)
#pragma unroll
        for (int b = 0; b < 4; b++) o[a][b] = make_float2(0.f, 0.f);
#pragma unroll 4
    for (int j = 0; j < 32; j++) {
        const float4 m0 = *(const float4*)(mt + j * 36 + r0);
        const float4 b0 = *(const float4*)(B + j * 32 + c0), b1 = *(const float4*)(B + j * 32 + c0 + 4);
        const float mr[4] = {m0.x, m0.y, m0.z, m0.w};
        const float2 bp[4] = {make_float2(b0.x, b0.y), make_float2(b0.z, b0.w), make_float2(b1.x, b1.y), make_float2(b1.z, b1.w)};
#pragma unroll
        for (int a = 0; a < 4; a++)
#pragma unroll
            for (int b = 0; b < 4; b++) o[a][b] = fma2(make_float2(mr[a], mr[a]), bp[b], o[a][b]);
    }
#pragma unroll
    for (int a = 0; a < 4; a++) {
        float* dst = t + (r0 + a) * 36 + c0;
        *(float4*)dst = make_float4(o[a][0].x, o[a][0].y, o[a][1].x, o[a][1].y);
        *(float4*)(dst + 4) = make_float4(o[a][2].x, o[a][2].y, o[a][3].x, o[a][3].y);
    }
}

// A Kronecker stage of row q by one warp: z in buf[from], result t in
// buf[from] too (pass 1 writes mt into buf[1 - from]). Both passes of a row
// are the one warp's, so only a warp barrier sits between them; the caller
// puts a block barrier before the result is read. (Tiles of 4 x 4 over two
// warps a row measured slower: the passes are bound by shared-memory
// wavefronts, three per 16 paired fmas here.)
template <int R>
__device__ __forceinline__ void kron_stage_row(PostSmem<R>& sm, int fa, int fb, int from, int q, int lane) {
    const int r0 = (lane & 7) * 4, c0 = (lane >> 3) * 8;
    kron_pass1(sm.kf[fa], sm.buf[from][q], sm.buf[1 - from][q], r0, c0);
    __syncwarp();
    kron_pass2(sm.buf[1 - from][q], sm.kf[fb], sm.buf[from][q], r0, c0);
}

// One conditioning logit chain (cond_weights, infer.rs:1640-1694): set s,
// output k: acc = fma(h[j], cond_v[j][k], acc) over j = s, s + 4, .., 764
// in order, from zero. The input is kept chain-major (element s + 4 n at
// hx[s * COND_LD + n]) and the weights one chain a row (row 8 s + k), so a
// chain's operands are 16-byte runs: four steps a load, loaded 16 steps
// ahead of the fma chain (two register buffers), which then waits on its
// own fmas alone.
__device__ __forceinline__ void cond_load16(const float* hr, const float* cr, int b, float4 (&hx)[4], float4 (&cx)[4]) {
#pragma unroll
    for (int e = 0; e < 4; e++) {
        hx[e] = *(const float4*)(hr + 16 * b + 4 * e);
        cx[e] = *(const float4*)(cr + 16 * b + 4 * e);
    }
}

__device__ __forceinline__ float cond_fma16(const float4 (&hx)[4], const float4 (&cx)[4], float acc) {
#pragma unroll
    for (int e = 0; e < 4; e++) {
        acc = __fmaf_rn(hx[e].x, cx[e].x, acc);
        acc = __fmaf_rn(hx[e].y, cx[e].y, acc);
        acc = __fmaf_rn(hx[e].z, cx[e].z, acc);
        acc = __fmaf_rn(hx[e].w, cx[e].w, acc);
    }
    return acc;
}

__device__ __forceinline__ float cond_chain(const float* hx, const float* cv, int set, int k) {
    const float* hr = hx + set * COND_LD;
    const float* cr = cv + (set * 8 + k) * COND_LD;
    float4 ha[4], ca[4], hb[4], cb[4];
    float acc = 0.f;
    cond_load16(hr, cr, 0, ha, ca);
#pragma unroll 1
    for (int b = 0; b < 12; b += 2) {
        cond_load16(hr, cr, b + 1, hb, cb);
        acc = cond_fma16(ha, ca, acc);
        if (b + 2 < 12) cond_load16(hr, cr, b + 2, ha, ca);
        acc = cond_fma16(hb, cb, acc);
    }
    return acc;
}

// dot16_combine over each half-warp (chain c in lane c of the half); the
// total is valid in lanes 0 and 16. Every lane of the warp must call it.
__device__ __forceinline__ float dot16_combine_half(float acc, int ln) {
    const unsigned F = 0xffffffffu;
    const int l = ln & 3;
    float a4 = __shfl_sync(F, acc, 4 + l, 16), a8 = __shfl_sync(F, acc, 8 + l, 16), a12 = __shfl_sync(F, acc, 12 + l, 16);
    float t = __fadd_rn(__fadd_rn(__fadd_rn(a8, a12), a4), acc);
    float t1 = __shfl_sync(F, t, 1, 16), t2 = __shfl_sync(F, t, 2, 16), t3 = __shfl_sync(F, t, 3, 16);
    return __fadd_rn(__fadd_rn(t, t1), __fadd_rn(t2, t3));
}

template <int POST_ROWS, int POST_THREADS = 64 * POST_ROWS>
__global__ void __launch_bounds__(POST_THREADS, 1) post_block_kernel(LayerW w, const float* o, const float* x1, const float* u,
                                                                   const float* gates, const int32_t* perm1,
                                                                   const int32_t* perm2, int M, float* xs) {
    static_assert(POST_ROWS * 768 % (4 * POST_THREADS) == 0, "whole batches of mHC items");
    pdl_launch_dependents();
    extern __shared__ __align__(16) int8_t post_raw[];
    PostSmem<POST_ROWS>& sm = *reinterpret_cast<PostSmem<POST_ROWS>*>(post_raw);
    const int tid = threadIdx.x, m0 = blockIdx.x * POST_ROWS;
    const int rows = min(POST_ROWS, M - m0);
    // group 0, before the predecessor is done: the layer's weights
    stage<POST_THREADS>(sm.post_norm, w.post_norm, 768 * 4, tid);
    for (int f = 0; f < 6; f++) stage<POST_THREADS>(sm.kf[f], w.kron[f], 4096, tid);
    stage<POST_THREADS>(sm.cond_v, w.cond_v, 32 * COND_LD * 4, tid);
    stage<POST_THREADS>(sm.cond_u, w.cond_u, 8 * 1024 * 4, tid);
    stage<POST_THREADS>(sm.d1, w.d1, 768 * 4, tid);
    stage<POST_THREADS>(sm.d2, w.d2, 4096, tid);
    stage<POST_THREADS>(sm.b2, w.b2, 4096, tid);
    stage<POST_THREADS>(sm.d3, w.d3, 4096, tid);
    stage<POST_THREADS>(sm.d4, w.d4, 768 * 4, tid);
    stage<POST_THREADS>(sm.pre_hada, w.pre_hada, 768 * 4, tid);
    stage<POST_THREADS>(sm.perm1, perm1, 4096, tid);
    stage<POST_THREADS>(sm.perm2, perm2, 4096, tid);
    asm volatile("cp.async.commit_group;\n" ::);
    pdl_wait();
    // group 1: the rows' o (into x2) and x1 (into buf[1], plain), gates
    for (int k = tid; k < POST_ROWS * 192; k += POST_THREADS) {
        const int q = k / 192, c = k % 192;
        const bool ok = q < rows;
        const size_t src = (size_t)(ok ? m0 + q : 0) * 768 + 4 * c;
        cp_async16(&sm.x2[q][4 * c], o + src, ok);
        cp_async16(&sm.buf[1][q][4 * c], x1 + src, ok);
    }
    for (int k = tid; k < POST_ROWS * 6; k += POST_THREADS) {
        const int q = k / 6, c = k % 6;
        const bool ok = q < rows;
        cp_async16(&sm.gates[q][4 * c], gates + (size_t)(ok ? m0 + q : 0) * 24 + 4 * c, ok);
    }
    asm volatile("cp.async.commit_group;\n" ::);
    asm volatile("cp.async.wait_group 0;\n" ::);
    __syncthreads();
    // zcn(o, post_norm): sixteen dot16 chains per row, a half-warp a row
    constexpr int NORM_THREADS = (POST_ROWS * 16 + 31) / 32 * 32;
    if (tid < NORM_THREADS) {
        const int q = tid >> 4;
        const float ch = q < POST_ROWS ? dot16_sq<768>(sm.x2[q], tid & 15) : 0.f;
        const float tot = dot16_combine_half(ch, tid & 31);
        if ((tid & 15) == 0 && q < POST_ROWS) sm.sc[q][0] = rinv(tot, 768);
    }
    __syncthreads();
    const float ga = __fdiv_rn(1.0f, __fadd_rn(lexpf(-w.attn_gate), 1.0f));
    for (int k = tid; k < POST_ROWS * 768; k += POST_THREADS) {
        int q = k / 768, c = k % 768;
        float tt = __fmul_rn(sm.x2[q][c], sm.sc[q][0]);
        float on = __fmaf_rn(tt, sm.post_norm[c], tt);
        sm.x2[q][c] = __fmaf_rn(on, ga, sm.buf[1][q][c]);
    }
    asm volatile("cp.async.wait_group 0;\n" ::);
    __syncthreads();
    if (tid < NORM_THREADS) {
        const int q = tid >> 4;
        const float ch = q < POST_ROWS ? dot16_sq<768>(sm.x2[q], tid & 15) : 0.f;
        const float tot = dot16_combine_half(ch, tid & 31);
        if ((tid & 15) == 0 && q < POST_ROWS) sm.sc[q][1] = rinv(tot, 768);
    }
    __syncthreads();
    // h2 = zcn(x2, pre_hada) into hs, z = h2 * d1 into buf[0]
    for (int k = tid; k < POST_ROWS * 768; k += POST_THREADS) {
        int q = k / 768, c = k % 768;
        float tt = __fmul_rn(sm.x2[q][c], sm.sc[q][1]);
        float h = __fmaf_rn(tt, sm.pre_hada[c], tt);
        sm.hs[q][(c & 3) * COND_LD + (c >> 2)] = h;
        sm.buf[0][q][pv_idx(c)] = __fmul_rn(h, sm.d1[c]);
    }
    for (int k = tid; k < POST_ROWS * 256; k += POST_THREADS) {
        int q = k >> 8, c = 768 + (k & 255);
        sm.buf[0][q][pv_idx(c)] = 0.f;
    }
    __syncthreads();
    // conditioning logits on warps 0..R-1 (4 accumulator sets by j % 4, fma
    // chains over j) while warps R..2R-1 run the first Kronecker stage
    // (t1 in buf[0])
    static_assert(2 * POST_ROWS * 32 <= POST_THREADS, "two warp sets");
    if (tid < POST_ROWS * 32) {
        const int q = tid >> 5, set = (tid >> 3) & 3, k = tid & 7;
        sm.part[q][tid & 31] = cond_chain(sm.hs[q], sm.cond_v, set, k);
    } else if (tid < 2 * POST_ROWS * 32) {
        kron_stage_row(sm, 0, 1, 0, (tid >> 5) - POST_ROWS, tid & 31);
    }
    __syncthreads();
    if (tid < POST_ROWS * 32) {
        // logits ((C + D) + B) + A, max, one libm exp per lane, the engine's
        // sum tree e7 + ((e6 + (e5 + e4)) + ((e3 + e2) + (e1 + e0)))
        const int q = tid >> 5, k = tid & 7;
        const float* pt = sm.part[q];
        float lg = __fadd_rn(__fadd_rn(__fadd_rn(pt[16 + k], pt[24 + k]), pt[8 + k]), pt[k]);
        float mx = lg;
#pragma unroll
        for (int off = 1; off < 8; off <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
        float e = lexpf(__fsub_rn(lg, mx));
        float ev[8];
#pragma unroll
        for (int qq = 0; qq < 8; qq++) ev[qq] = __shfl_sync(0xffffffffu, e, qq);
        float sum = __fadd_rn(ev[7], __fadd_rn(__fadd_rn(ev[6], __fadd_rn(ev[5], ev[4])), __fadd_rn(__fadd_rn(ev[3], ev[2]), __fadd_rn(ev[1], ev[0]))));
        if ((tid & 31) < 8) sm.wk[q][k] = __fmul_rn(e, __fdiv_rn(1.0f, sum));
    }
    __syncthreads();
    // z = fma(t1[perm1[j]], cond[j] * d2[j], b2[j]) with cond = 1 + sum_k w_k u_k,
    // then SiLU; into buf[1]. Whole strides of j take every row; the last,
    // partial stride's (j, row) items are spread over all threads, RT rows
    // a thread, so no warp runs a third stride alone.
    auto silu_item = [&](int j, int q0, int nq) {
        float cu[8];
#pragma unroll
        for (int kk = 0; kk < 8; kk++) cu[kk] = sm.cond_u[kk * 1024 + j];
        const float d2 = sm.d2[j], b2 = sm.b2[j];
        const int src = pv_idx(sm.perm1[j]), dst = pv_idx(j);
#pragma unroll
        for (int qq = 0; qq < POST_ROWS; qq++) {
            if (qq >= nq) break;
            const int q = q0 + qq;
            float cnd = 1.0f;
#pragma unroll
            for (int kk = 0; kk < 8; kk++) cnd = __fmaf_rn(cu[kk], sm.wk[q][kk], cnd);
            float zz = __fmaf_rn(sm.buf[0][q][src], __fmul_rn(cnd, d2), b2);
            sm.buf[1][q][dst] = __fdiv_rn(zz, __fadd_rn(nexp(-zz), 1.0f));
        }
    };
    {
        constexpr int FULL = 1024 / POST_THREADS * POST_THREADS, TAIL = 1024 - FULL;
        for (int j = tid; j < FULL; j += POST_THREADS) silu_item(j, 0, POST_ROWS);
        if constexpr (TAIL > 0) {
            // POST_THREADS / TAIL thread sets, each taking RT rows of the tail
            constexpr int SETS = POST_THREADS / (TAIL > 0 ? TAIL : 1), RT = (POST_ROWS + SETS - 1) / SETS;
            const int set = tid / (TAIL > 0 ? TAIL : 1), q0 = set * RT;
            if (set < SETS && q0 < POST_ROWS) silu_item(FULL + tid % TAIL, q0, min(RT, POST_ROWS - q0));
        }
    }
    __syncthreads();
    if (tid < POST_ROWS * 32) kron_stage_row(sm, 2, 3, 1, tid >> 5, tid & 31);  // t2 in buf[1]
    __syncthreads();
    for (int j = tid; j < 1024; j += POST_THREADS) {
        const float d3 = sm.d3[j];
        const int src = pv_idx(sm.perm2[j]), dst = pv_idx(j);
#pragma unroll
        for (int q = 0; q < POST_ROWS; q++) sm.buf[0][q][dst] = __fmul_rn(sm.buf[1][q][src], d3);
    }
    __syncthreads();
    // mHC write (infer.rs:1587-1606): y = x2 + mlp - u, stream a =
    // y * hpost[a] + sum_b old[b] * hres[a][b]. Four (row, channel) items a
    // thread per round, each round's loads (four old streams and u an item)
    // issued before the previous round's arithmetic (the first round's
    // before the last Kronecker stage).
    constexpr int ITEMS = POST_ROWS * 768 / POST_THREADS, BATCH = 4;
    static_assert(ITEMS % BATCH == 0, "item batches");
    float cur[BATCH][5], nxt[BATCH][5];  // per item the four old streams, then u
#define POST_LOAD_OLD(dst, it0)                                                                       \
    _Pragma("unroll") for (int e = 0; e < BATCH; e++) {                                               \
        const int k = tid + ((it0) + e) * POST_THREADS, q = k / 768, ch = k % 768;                    \
        const size_t mq = (size_t)(m0 + (q < rows ? q : 0));                                          \
        const float* xr = xs + mq * 3072 + ch;                                                        \
        _Pragma("unroll") for (int b = 0; b < 4; b++) dst[e][b] = xr[b * 768];                        \
        dst[e][4] = u[mq * 768 + ch];                                                                 \
    }
    POST_LOAD_OLD(cur, 0)  // in flight during the last Kronecker stage
    if (tid < POST_ROWS * 32) kron_stage_row(sm, 4, 5, 0, tid >> 5, tid & 31);  // t3 in buf[0]
    asm volatile("cp.async.wait_group 0;\n" ::);
    __syncthreads();
#pragma unroll
    for (int it0 = 0; it0 < ITEMS; it0 += BATCH) {
        if (it0 + BATCH < ITEMS) {
            POST_LOAD_OLD(nxt, it0 + BATCH)
        }
#pragma unroll
        for (int e = 0; e < BATCH; e++) {
            const int k = tid + (it0 + e) * POST_THREADS, q = k / 768, ch = k % 768;
            if (q >= rows) continue;
            const float* gr = sm.gates[q];
            float mlp = __fmul_rn(sm.buf[0][q][pv_idx(ch)], sm.d4[ch]);
            float y = __fsub_rn(__fadd_rn(sm.x2[q][ch], mlp), cur[e][4]);
            float* xr = xs + (size_t)(m0 + q) * 3072 + ch;
#pragma unroll
            for (int a = 0; a < 4; a++) {
                float v = __fmul_rn(y, gr[a]);
#pragma unroll
                for (int b = 0; b < 4; b++) v = __fmaf_rn(cur[e][b], gr[4 + a * 4 + b], v);
                xr[a * 768] = v;
            }
        }
#pragma unroll
        for (int e = 0; e < BATCH; e++)
#pragma unroll
            for (int b = 0; b < 5; b++) cur[e][b] = nxt[e][b];
    }
#undef POST_LOAD_OLD
}

// The same post block for small batches: one row per CTA of 512 threads,
// the layer's small weights staged into shared memory as post_block_kernel
// stages them (before the wait on the predecessor), every thread on the one
// row. A Kronecker pass runs on warps 1-4, a 2 x 4 tile of outputs a
// thread (mt stored transposed, as kron_native keeps it), while warp 0's
// conditioning chains may still run. Every float op, and its order, is
// that of post_block_kernel.
constexpr int POST_ROW_THREADS = 512;
struct PostRowSmem {
    float kf[6][1024];
    __align__(16) float cond_v[32 * COND_LD];
    float cond_u[8 * 1024];
    float d1[768], d2[1024], b2[1024], d3[1024], d4[768];
    float post_norm[768], pre_hada[768];
    int perm1[1024], perm2[1024];
    float x2[768];
    __align__(16) float hb[4 * COND_LD];  // the conditioning input, chain-major
    float zb[1024], mb[1024], tb[1024];
    float x1[768], ub[768], xold[3072];  // the row's residual, u and streams
    float part[32], sc[2], wk[8], gr[24];
};
extern const size_t POST_ROW_SMEM = sizeof(PostRowSmem);

// The one-row Kronecker passes: 128 threads, each a 2 x 4 tile (rows r0,
// r0 + 1; columns c0..c0 + 3), one 8-byte and one 16-byte shared load per
// four paired fmas; every output one fma chain over j = 0..31 from zero.
// Pass 1: mt[c][r] = sum_j A[j][r] z[j][c] (stored transposed).
__device__ __forceinline__ void kron_row_pass1(const float* A, const float* z, float* mt, int r0, int c0) {
    float2 o[2][2];
#pragma unroll
    for (int a = 0; a < 2; a++) o[a][0] = o[a][1] = make_float2(0.f, 0.f);
#pragma unroll 8
    for (int j = 0; j < 32; j++) {
        const float2 a2 = *(const float2*)(A + j * 32 + r0);
        const float4 z4 = *(const float4*)(z + j * 32 + c0);
        const float ar[2] = {a2.x, a2.y};
#pragma unroll
        for (int a = 0; a < 2; a++) {
            o[a][0] = fma2(make_float2(ar[a], ar[a]), make_float2(z4.x, z4.y), o[a][0]);
            o[a][1] = fma2(make_float2(ar[a], ar[a]), make_float2(z4.z, z4.w), o[a][1]);
        }
    }
    *(float2*)(mt + c0 * 32 + r0) = make_float2(o[0][0].x, o[1][0].x);
    *(float2*)(mt + (c0 + 1) * 32 + r0) = make_float2(o[0][0].y, o[1][0].y);
    *(float2*)(mt + (c0 + 2) * 32 + r0) = make_float2(o[0][1].x, o[1][1].x);
    *(float2*)(mt + (c0 + 3) * 32 + r0) = make_float2(o[0][1].y, o[1][1].y);
}

// Pass 2: t[r][c] = sum_j mt[j][r] B[j][c].
__device__ __forceinline__ void kron_row_pass2(const float* mt, const float* B, float* t, int r0, int c0) {
    float2 o[2][2];
#pragma unroll
    for (int a = 0; a < 2; a++) o[a][0] = o[a][1] = make_float2(0.f, 0.f);
#pragma unroll 8
    for (int j = 0; j < 32; j++) {
        const float2 m2 = *(const float2*)(mt + j * 32 + r0);
        const float4 b4 = *(const float4*)(B + j * 32 + c0);
        const float mr[2] = {m2.x, m2.y};
#pragma unroll
        for (int a = 0; a < 2; a++) {
            o[a][0] = fma2(make_float2(mr[a], mr[a]), make_float2(b4.x, b4.y), o[a][0]);
            o[a][1] = fma2(make_float2(mr[a], mr[a]), make_float2(b4.z, b4.w), o[a][1]);
        }
    }
#pragma unroll
    for (int a = 0; a < 2; a++)
        *(float4*)(t + (r0 + a) * 32 + c0) = make_float4(o[a][0].x, o[a][0].y, o[a][1].x, o[a][1].y);
}

// The one-row post block of row m by a CTA of POST_ROW_THREADS threads
// with PostRowSmem as its dynamic shared memory.
__device__ __forceinline__ void post_row_row(const LayerW& w, const float* o, const float* x1, const float* u, const float* gates,
                                             const int32_t* perm1, const int32_t* perm2, float* xs, int m) {
    pdl_launch_dependents();
    extern __shared__ __align__(16) int8_t post_row_raw[];
    PostRowSmem& sm = *reinterpret_cast<PostRowSmem*>(post_row_raw);
    const int tid = threadIdx.x;
    // the Kronecker passes run on warps 1-4 (warp 0 has the conditioning chains)
    const int kt = tid - 32, r0 = 2 * (kt & 15), c0 = 4 * (kt >> 4);
    const bool kw = kt >= 0 && kt < 128;
    for (int f = 0; f < 6; f++) stage<POST_ROW_THREADS>(sm.kf[f], w.kron[f], 4096, tid);
    stage<POST_ROW_THREADS>(sm.cond_v, w.cond_v, 32 * COND_LD * 4, tid);
    stage<POST_ROW_THREADS>(sm.cond_u, w.cond_u, 8 * 1024 * 4, tid);
    stage<POST_ROW_THREADS>(sm.d1, w.d1, 768 * 4, tid);
    stage<POST_ROW_THREADS>(sm.d2, w.d2, 4096, tid);
    stage<POST_ROW_THREADS>(sm.b2, w.b2, 4096, tid);
    stage<POST_ROW_THREADS>(sm.d3, w.d3, 4096, tid);
    stage<POST_ROW_THREADS>(sm.d4, w.d4, 768 * 4, tid);
    stage<POST_ROW_THREADS>(sm.post_norm, w.post_norm, 768 * 4, tid);
    stage<POST_ROW_THREADS>(sm.pre_hada, w.pre_hada, 768 * 4, tid);
    stage<POST_ROW_THREADS>(sm.perm1, perm1, 4096, tid);
    stage<POST_ROW_THREADS>(sm.perm2, perm2, 4096, tid);
    asm volatile("cp.async.commit_group;\n" ::);
    pdl_wait();
    // the row's inputs in one round of copies: o, the residual x1, u, the
    // four streams the mHC write reads, the gates
    float* xr = xs + (size_t)m * 3072;
    stage<POST_ROW_THREADS>(sm.x2, o + (size_t)m * 768, 768 * 4, tid);
    stage<POST_ROW_THREADS>(sm.x1, x1 + (size_t)m * 768, 768 * 4, tid);
    stage<POST_ROW_THREADS>(sm.ub, u + (size_t)m * 768, 768 * 4, tid);
    stage<POST_ROW_THREADS>(sm.xold, xr, 3072 * 4, tid);
    if (tid < 24) sm.gr[tid] = gates[(size_t)m * 24 + tid];
    asm volatile("cp.async.commit_group;\n" ::);
    asm volatile("cp.async.wait_group 0;\n" ::);
    __syncthreads();
    // zcn(o, post_norm): sixteen dot16 chains
    if (tid < 16) sm.part[tid] = dot16_sq<768>(sm.x2, tid);
    __syncthreads();
    if (tid == 0) sm.sc[0] = rinv(dot16_combine(sm.part), 768);
    __syncthreads();
    const float ga = __fdiv_rn(1.0f, __fadd_rn(lexpf(-w.attn_gate), 1.0f));
    for (int c = tid; c < 768; c += POST_ROW_THREADS) {
        float tt = __fmul_rn(sm.x2[c], sm.sc[0]);
        float on = __fmaf_rn(tt, sm.post_norm[c], tt);
        sm.x2[c] = __fmaf_rn(on, ga, sm.x1[c]);
    }
    __syncthreads();
    if (tid < 16) sm.part[tid] = dot16_sq<768>(sm.x2, tid);
    __syncthreads();
    if (tid == 0) sm.sc[1] = rinv(dot16_combine(sm.part), 768);
    __syncthreads();
    // h2 = zcn(x2, pre_hada), z = h2 * d1 (zero past 768)
    for (int c = tid; c < 1024; c += POST_ROW_THREADS) {
        if (c < 768) {
            float tt = __fmul_rn(sm.x2[c], sm.sc[1]);
            float h = __fmaf_rn(tt, sm.pre_hada[c], tt);
            sm.hb[(c & 3) * COND_LD + (c >> 2)] = h;
            sm.zb[c] = __fmul_rn(h, sm.d1[c]);
        } else {
            sm.zb[c] = 0.f;
        }
    }
    __syncthreads();
    // conditioning logits: 4 accumulator sets by j % 4, fma chains over j
    if (tid < 32) {
        const int set = (tid >> 3) & 3, k = tid & 7;
        sm.part[tid] = cond_chain(sm.hb, sm.cond_v, set, k);
        __syncwarp();
        // logits ((C + D) + B) + A, max, one libm exp per lane, the engine's
        // sum tree e7 + ((e6 + (e5 + e4)) + ((e3 + e2) + (e1 + e0)))
        float lg = __fadd_rn(__fadd_rn(__fadd_rn(sm.part[16 + k], sm.part[24 + k]), sm.part[8 + k]), sm.part[k]);
        float mx = lg;
#pragma unroll
        for (int off = 1; off < 8; off <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
        float e = lexpf(__fsub_rn(lg, mx));
        float ev[8];
#pragma unroll
        for (int qq = 0; qq < 8; qq++) ev[qq] = __shfl_sync(0xffffffffu, e, qq);
        float sum = __fadd_rn(ev[7], __fadd_rn(__fadd_rn(ev[6], __fadd_rn(ev[5], ev[4])), __fadd_rn(__fadd_rn(ev[3], ev[2]), __fadd_rn(ev[1], ev[0]))));
        if (tid < 8) sm.wk[k] = __fmul_rn(e, __fdiv_rn(1.0f, sum));
    }
    // stage 1: t1 = (A0^T z) A1
    if (kw) kron_row_pass1(sm.kf[0], sm.zb, sm.mb, r0, c0);
    __syncthreads();
    if (kw) kron_row_pass2(sm.mb, sm.kf[1], sm.tb, r0, c0);
    __syncthreads();
    // z = fma(t1[perm1[j]], cond[j] * d2[j], b2[j]), cond = 1 + sum_k w_k u_k, then SiLU
    for (int j = tid; j < 1024; j += POST_ROW_THREADS) {
        float cnd = 1.0f;
#pragma unroll
        for (int kk = 0; kk < 8; kk++) cnd = __fmaf_rn(sm.cond_u[kk * 1024 + j], sm.wk[kk], cnd);
        float zz = __fmaf_rn(sm.tb[sm.perm1[j]], __fmul_rn(cnd, sm.d2[j]), sm.b2[j]);
        sm.zb[j] = __fdiv_rn(zz, __fadd_rn(nexp(-zz), 1.0f));
    }
    __syncthreads();
    if (kw) kron_row_pass1(sm.kf[2], sm.zb, sm.mb, r0, c0);
    __syncthreads();
    if (kw) kron_row_pass2(sm.mb, sm.kf[3], sm.tb, r0, c0);
    __syncthreads();
    for (int j = tid; j < 1024; j += POST_ROW_THREADS) sm.zb[j] = __fmul_rn(sm.tb[sm.perm2[j]], sm.d3[j]);
    __syncthreads();
    if (kw) kron_row_pass1(sm.kf[4], sm.zb, sm.mb, r0, c0);
    __syncthreads();
    if (kw) kron_row_pass2(sm.mb, sm.kf[5], sm.tb, r0, c0);
    __syncthreads();
    // mHC write (infer.rs:1587-1606): y = x2 + mlp - u, stream a =
    // y * hpost[a] + sum_b old[b] * hres[a][b]
    for (int ch = tid; ch < 768; ch += POST_ROW_THREADS) {
        float mlp = __fmul_rn(sm.tb[ch], sm.d4[ch]);
        float y = __fsub_rn(__fadd_rn(sm.x2[ch], mlp), sm.ub[ch]);
        float old[4];
#pragma unroll
        for (int bb = 0; bb < 4; bb++) old[bb] = sm.xold[bb * 768 + ch];
#pragma unroll
        for (int aa = 0; aa < 4; aa++) {
            float v = __fmul_rn(y, sm.gr[aa]);
#pragma unroll
            for (int bb = 0; bb < 4; bb++) v = __fmaf_rn(old[bb], sm.gr[4 + aa * 4 + bb], v);
            xr[aa * 768 + ch] = v;
        }
    }
}

__global__ void __launch_bounds__(POST_ROW_THREADS, 1) post_row_kernel(LayerW w, const float* o, const float* x1, const float* u,
                                                                 const float* gates, const int32_t* perm1, const int32_t* perm2,
                                                                 float* xs) {
    post_row_row(w, o, x1, u, gates, perm1, perm2, xs, blockIdx.x);
}

// The post block of one layer and the mHC read of the next for the same
// row, one CTA a row (batches of at most one row an SM): one launch fewer a
// layer. The post block has staged this layer's u, x1 and gates before the
// mHC read overwrites those buffers with the next layer's, and the row's
// new streams it wrote to xs are visible to the CTA's threads after the
// barrier. Each value is computed as post_row_kernel and mhc_read_kernel
// compute it.
__global__ void __launch_bounds__(POST_ROW_THREADS, 1) post_mhc_kernel(LayerW w, const float* o, const float* x1, const float* u,
                                                                 const float* gates, const int32_t* perm1, const int32_t* perm2,
                                                                 float* xs, LayerW wn, int lane_next, float* un, float* pn,
                                                                 const float* ekv, const float* evals, float* x1n, int8_t* act,
                                                                 float* sx) {
    post_row_row(w, o, x1, u, gates, perm1, perm2, xs, blockIdx.x);
    __syncthreads();
    if (threadIdx.x < MHC_THREADS) mhc_read_row<1, true>(wn, lane_next, xs, un, pn, ekv, evals, x1n, act, sx, blockIdx.x);
}

void launch_post_block(LayerW w, const float* o, const float* x1, const float* u, const float* gates, const int32_t* perm1,
                       const int32_t* perm2, int M, float* xs, cudaStream_t st) {
    COUNT_LAUNCH();
    // The fewest rows a CTA (1, 2, 4 or 7) whose CTAs fit one wave of one
    // CTA an SM; seven (the most shared memory allows) past that.
    const int sms = sm_count();
    if (M <= sms) {
        launch_pdl(post_row_kernel, dim3(M), dim3(POST_ROW_THREADS), POST_ROW_SMEM, st, w, o, x1, u, gates, perm1, perm2, xs);
    } else if (cdiv(M, 2) <= sms) {
        launch_pdl(post_block_kernel<2>, dim3(cdiv(M, 2)), dim3(128), sizeof(PostSmem<2>), st, w, o, x1, u, gates, perm1, perm2, M, xs);
    } else if (cdiv(M, 4) <= sms) {
        launch_pdl(post_block_kernel<4>, dim3(cdiv(M, 4)), dim3(256), sizeof(PostSmem<4>), st, w, o, x1, u, gates, perm1, perm2, M, xs);
    } else {
        launch_pdl(post_block_kernel<7>, dim3(cdiv(M, 7)), dim3(448), sizeof(PostSmem<7>), st, w, o, x1, u, gates, perm1, perm2, M, xs);
    }
}

cudaError_t launch_post_mhc(LayerW w, const float* o, const float* x1, const float* u, const float* gates, const int32_t* perm1,
                            const int32_t* perm2, int M, float* xs, LayerW wn, int lane_next, float* un, float* pn, const float* ekv,
                            const float* evals, float* x1n, int8_t* act, float* sx, cudaStream_t st) {
    if (M < 1 || M > sm_count()) return cudaErrorInvalidValue;
    COUNT_LAUNCH();
    launch_pdl(post_mhc_kernel, dim3(M), dim3(POST_ROW_THREADS), POST_ROW_SMEM, st, w, o, x1, u, gates, perm1, perm2, xs, wn, lane_next,
               un, pn, ekv, evals, x1n, act, sx);
    return cudaSuccess;
}

cudaError_t post_block_init() {
    cudaFuncSetAttribute(post_mhc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)POST_ROW_SMEM);
    cudaFuncSetAttribute(post_block_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(PostSmem<2>));
    cudaFuncSetAttribute(post_block_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(PostSmem<4>));
    return cudaFuncSetAttribute(post_block_kernel<7>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(PostSmem<7>));
}

// ------------------------------------------------------------ final norm

// infer.rs:1214-1225: lane mean ((x0 + x1) + x2 + x3) * 0.25, then the final
// ZC-RMSNorm, for each sequence's last row (or every row).
__global__ void final_hidden_kernel(const float* xs, const float* fnorm, int T, int all_rows, float* h) {
    pdl_launch_dependents();
    pdl_wait();
    __shared__ float mean[768];
    __shared__ float part[16];
    __shared__ float r_s;
    const int q = blockIdx.x, tid = threadIdx.x;
    const int m = all_rows ? q : q * T + T - 1;
    const float* x = xs + (size_t)m * 3072;
    for (int ch = tid; ch < 768; ch += 256)
        mean[ch] = __fmul_rn(__fadd_rn(__fadd_rn(__fadd_rn(x[ch], x[768 + ch]), x[1536 + ch]), x[2304 + ch]), 0.25f);
    __syncthreads();
    if (tid < 16) part[tid] = dot16_sq<768>(mean, tid);
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
    launch_pdl(final_hidden_kernel, dim3(all_rows ? S * T : S), dim3(256), 0, st, xs, final_norm, T, all_rows, h);
}

// ----------------------------------------------------------------- RoPE

// infer.rs:1716-1744: table rows (sincosf of freq * pos, tabulated on the
// host with the reference's f64 libm stand-in) for a chunk, or for a single
// token right after the newest position the angle-addition recurrence.
__global__ void rope_rows_kernel(const float* tc, const float* tsn, const float* sd, const float* cd, const int32_t* p0p, int T, int recur,
                                 float* state, float* cosr, float* sinr) {
    pdl_launch_dependents();
    pdl_wait();
    const int p0 = *p0p;
    int i = blockIdx.x, f = threadIdx.x;
    if (f >= 24) return;
    float cv, sv;
    if (recur) {
        const float* r = state + (size_t)((p0 - 1) % ROPE_RING) * 48;
        float c0 = r[f], s0 = r[24 + f];
        cv = __fmaf_rn(-sd[f], s0, __fmul_rn(cd[f], c0));
        sv = __fmaf_rn(sd[f], c0, __fmul_rn(cd[f], s0));
    } else {
        cv = tc[(size_t)(p0 + i) * 24 + f];
        sv = tsn[(size_t)(p0 + i) * 24 + f];
    }
    cosr[i * 24 + f] = cv;
    sinr[i * 24 + f] = sv;
    float* w = state + (size_t)((p0 + i) % ROPE_RING) * 48;
    w[f] = cv;
    w[24 + f] = sv;
}

void launch_rope_rows(const float* table_cos, const float* table_sin, const float* sd, const float* cd, const int32_t* p0p, int T,
                      int recur, float* state, float* cosr, float* sinr, cudaStream_t st) {
    COUNT_LAUNCH();
    launch_pdl(rope_rows_kernel, dim3(T), dim3(32), 0, st, table_cos, table_sin, sd, cd, p0p, T, recur, state, cosr, sinr);
}

// Positions fed so far, advanced on the device so a captured step replays
// at any position.
__global__ void advance_len_kernel(int32_t* len, int T) {
    pdl_launch_dependents();
    pdl_wait(); *len += T; }

void launch_advance_len(int32_t* len, int T, cudaStream_t st) {
    COUNT_LAUNCH();
    launch_pdl(advance_len_kernel, dim3(1), dim3(1), 0, st, len, T);
}

// Holds the stream for `ns` nanoseconds (one thread, sleeping), so that the
// launches queued behind it start back to back: per-site event timing then
// sees kernel time, not the host's launch rate.
__global__ void hold_kernel(unsigned long long ns) {
    pdl_launch_dependents();
    pdl_wait();
    unsigned long long t0, t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
    do {
        __nanosleep(1000);
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    } while (t - t0 < ns);
}

void launch_hold(unsigned long long ns, cudaStream_t st) {
    COUNT_LAUNCH();
    launch_pdl(hold_kernel, dim3(1), dim3(1), 0, st, ns);
}

// ------------------------------------------------------- masked argmax

// crates/needle-engine/src/agent.rs:1114-1127: banned ids read -1e30, then
// the first index of the maximum.
__global__ void masked_argmax_kernel(const float* logits, int V, const uint8_t* allow, int32_t* next) {
    pdl_launch_dependents();
    pdl_wait();
    __shared__ float bv[32];
    __shared__ int bi[32];
    const int s = blockIdx.x, tid = threadIdx.x;
    const float* x = logits + (size_t)s * V;
    const uint8_t* al = allow ? allow + (size_t)s * ((V + 7) / 8) : nullptr;
    float best = -INFINITY;
    int idx = 0x7fffffff;
    // whole 8-id blocks: two float4 loads and one mask byte per block
    const int nb = (V % 8 == 0) ? V / 8 : 0;
    for (int q = tid; q < nb; q += blockDim.x) {
        float4 a = *(const float4*)(x + 8 * q), b = *(const float4*)(x + 8 * q + 4);
        unsigned bits = al ? al[q] : 0xffu;
        float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
        for (int e = 0; e < 8; e++) {
            float ve = ((bits >> e) & 1) ? v[e] : -1e30f;
            if (ve > best) { best = ve; idx = 8 * q + e; }  // ascending ids: first index wins ties
        }
    }
    for (int k = nb * 8 + tid; k < V; k += blockDim.x) {
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
    launch_pdl(masked_argmax_kernel, dim3(S), dim3(256), 0, st, logits, V, allow, next);
}

// ----------------------------------------------------------- call sampler
//
// The statistics and candidate order the agent's grammar-constrained call
// step starts from, per sequence (agent.rs:295-343): softmax_stats
// (agent.rs:1241-1252) over the logits with the step's bans, then the
// unmasked candidates by logit (lowest id first on ties) after the call
// step's further bans, the first k of them. Two kernels, the row's logits
// read from L2 a few times each:
//   * cand_select_kernel, one 256-thread CTA per sequence: the max
//     (order-free: f32::max as the reference's platform has it), the live
//     count and each thread's smallest 48-bit key (~orderable(logit) << 16
//     | id, ascending in the reference's order); the k-th smallest of those
//     256 keys bounds the candidates (at least k keys lie at or below it,
//     usually a couple of hundred in all), which are gathered into shared
//     memory and sorted by a bitonic network; should more than CAND_BUF
//     qualify, the k smallest are drawn one at a time instead;
//     it also writes engine_expf(v - max) of every element of the whole
//     groups of four to a lane-major scratch row (lane j: elements 4i + j);
//   * cand_sum_kernel, one warp per sequence: lanes 0-3 add lane j's exps
//     in i order, the reference's four lane chains (lane_exp_sums,
//     agent.rs:1147-1198), each a dependent run of V/4 f32 adds, fed from
//     the scratch row by cp.async double buffering.
constexpr int CAND_MAXK = 128, CAND_BUF = 1024, CSEL_THREADS = 256;

// agent.rs:1130-1145: the engine's own f32 exp (its constants).
__device__ __forceinline__ float engine_expf(float x) {
    x = fminf(fmaxf(x, -88.37626f), 88.37626f);
    const float n = rintf(__fmul_rn(x, 1.44269504088896340736f));
    x = __fmaf_rn(n, -0.6933594f, x);
    x = __fmaf_rn(n, 2.1219444e-4f, x);
    float p = 1.9875691e-4f;
    p = __fmaf_rn(p, x, 1.3981999e-3f);
    p = __fmaf_rn(p, x, 8.333452e-3f);
    p = __fmaf_rn(p, x, 4.1665796e-2f);
    p = __fmaf_rn(p, x, 1.6666665e-1f);
    p = __fmaf_rn(p, x, 0.5f);
    const float y = __fmaf_rn(__fmul_rn(x, x), p, x);
    const float two_n = __uint_as_float((unsigned)((int)n + 127) << 23);
    return __fmaf_rn(two_n, y, two_n);
}

// Ascending 48-bit key of (logit descending, id ascending); -0 and +0 are
// the same logit, as partial_cmp has them.
__device__ __forceinline__ unsigned long long cand_key(float v, int i) {
    if (v == 0.f) v = 0.f;
    unsigned u = __float_as_uint(v);
    u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return ((unsigned long long)(~u) << 16) | (unsigned)i;
}

__device__ __forceinline__ bool bit_clear(const uint8_t* bits, int i) { return bits && !((bits[i >> 3] >> (i & 7)) & 1); }

// f32::max as the reference's platform computes it (aarch64 FMAXNM): equal
// values keep +0 over -0, so the result does not depend on the order.
__device__ __forceinline__ float fmaxnm(float a, float b) {
    if (a > b) return a;
    if (b > a) return b;
    return signbit(a) ? b : a;
}

__device__ __forceinline__ unsigned long long umin64(unsigned long long a, unsigned long long b) { return a < b ? a : b; }
__device__ __forceinline__ unsigned long long umax64(unsigned long long a, unsigned long long b) { return a < b ? b : a; }

// The logit of element i as the row's bans leave it (-1e30 when banned).
__device__ __forceinline__ float cand_logit(const float* x, const uint8_t* a1, const uint8_t* a2, int i) {
    return (bit_clear(a1, i) || bit_clear(a2, i)) ? -1e30f : __ldg(x + i);
}

constexpr int CAND_UNROLL = 8;  // elements a thread has in flight together

__global__ void __launch_bounds__(CSEL_THREADS) cand_select_kernel(const float* logits, int V, const uint8_t* allow,
                                                                   const uint8_t* allow_order, int k, int32_t* ids,
                                                                   float* mo, int32_t* live_out, float* ex) {
    pdl_launch_dependents();
    pdl_wait();
    __shared__ unsigned long long sk[CAND_BUF];
    __shared__ float redf[CSEL_THREADS / 32];
    __shared__ int redi[CSEL_THREADS / 32];
    __shared__ unsigned long long s_t0;
    __shared__ int s_count;
    const unsigned FULL = 0xffffffffu;
    const int s = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const float* x = logits + (size_t)s * V;
    const size_t mb = (size_t)(V + 7) / 8;
    const uint8_t* a1 = allow ? allow + (size_t)s * mb : nullptr;
    const uint8_t* a2 = allow_order ? allow_order + (size_t)s * mb : nullptr;
    constexpr int STEP = CSEL_THREADS * CAND_UNROLL;
    // the max
    float mx = -INFINITY;
    for (int base = 0; base < V; base += STEP) {
        float vv[CAND_UNROLL];
#pragma unroll
        for (int u = 0; u < CAND_UNROLL; u++) {
            const int i = base + CSEL_THREADS * u + tid;
            vv[u] = i < V ? cand_logit(x, a1, nullptr, i) : -INFINITY;
        }
#pragma unroll
        for (int u = 0; u < CAND_UNROLL; u++) mx = fmaxnm(mx, vv[u]);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) mx = fmaxnm(mx, __shfl_xor_sync(FULL, mx, o));
    if (lane == 0) redf[warp] = mx;
    if (tid == 0) s_count = 0;
    __syncthreads();
    float m = redf[0];
    for (int w = 1; w < CSEL_THREADS / 32; w++) m = fmaxnm(m, redf[w]);
    // the exps (lane-major: element 4i + j at ex[j][i]); with the order
    // bans, the live count and each thread's best key
    const int Q = V / 4;
    float* er = ex + (size_t)s * 4 * Q;
    int nl = 0;
    unsigned long long best = ~0ull;
    for (int base = 0; base < V; base += STEP) {
        float vv[CAND_UNROLL];
        bool b2[CAND_UNROLL];
#pragma unroll
        for (int u = 0; u < CAND_UNROLL; u++) {
            const int i = base + CSEL_THREADS * u + tid;
            vv[u] = i < V ? cand_logit(x, a1, nullptr, i) : -INFINITY;
            b2[u] = i < V && bit_clear(a2, i);
        }
#pragma unroll
        for (int u = 0; u < CAND_UNROLL; u++) {
            const int i = base + CSEL_THREADS * u + tid;
            if (i < 4 * Q) er[(i & 3) * Q + (i >> 2)] = engine_expf(__fsub_rn(vv[u], m));
            if (i < V && !b2[u] && vv[u] > -1e30f) {
                nl++;
                best = umin64(best, cand_key(vv[u], i));
            }
        }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) nl += __shfl_xor_sync(FULL, nl, o);
    if (lane == 0) redi[warp] = nl;
    __syncthreads();
    int live = redi[0];
    for (int w = 1; w < CSEL_THREADS / 32; w++) live += redi[w];
    const int K = min(k, live);
    int32_t* out = ids + (size_t)s * k;
    if (K > 0) {
        // the threads' best keys sorted (shuffles below stride 32, shared
        // memory above); at least K keys lie at or below the K-th of them
        unsigned long long key = best;
#pragma unroll
        for (int size = 2; size <= CSEL_THREADS; size <<= 1) {
            const bool asc = (tid & size) == 0;
#pragma unroll
            for (int stride = size >> 1; stride > 0; stride >>= 1) {
                unsigned long long o;
                if (stride >= 32) {
                    __syncthreads();
                    sk[tid] = key;
                    __syncthreads();
                    o = sk[tid ^ stride];
                } else {
                    o = __shfl_xor_sync(FULL, key, stride);
                }
                key = (((tid & stride) == 0) == asc) ? umin64(key, o) : umax64(key, o);
            }
        }
        if (tid == K - 1) s_t0 = key;
        __syncthreads();
        const unsigned long long t0 = s_t0;
        // the candidates: every live key at or below t0
        for (int base = 0; base < V; base += STEP) {
            float vv[CAND_UNROLL];
#pragma unroll
            for (int u = 0; u < CAND_UNROLL; u++) {
                const int i = base + CSEL_THREADS * u + tid;
                vv[u] = i < V ? cand_logit(x, a1, a2, i) : -INFINITY;
            }
#pragma unroll
            for (int u = 0; u < CAND_UNROLL; u++) {
                const int i = base + CSEL_THREADS * u + tid;
                unsigned long long kk = 0;
                bool take = false;
                if (vv[u] > -1e30f) {
                    kk = cand_key(vv[u], i);
                    take = kk <= t0;
                }
                const unsigned bal = __ballot_sync(FULL, take);
                int pos0 = 0;
                if (lane == 0 && bal) pos0 = atomicAdd(&s_count, __popc(bal));
                pos0 = __shfl_sync(FULL, pos0, 0);
                const int pos = pos0 + __popc(bal & ((1u << lane) - 1u));
                if (take && pos < CAND_BUF) sk[pos] = kk;
            }
        }
        __syncthreads();
        const int C = s_count;
        if (C <= CAND_BUF) {
            int n = 2;
            while (n < C) n <<= 1;
            for (int j = C + tid; j < n; j += CSEL_THREADS) sk[j] = ~0ull;
            for (int size = 2; size <= n; size <<= 1)
                for (int stride = size >> 1; stride > 0; stride >>= 1) {
                    __syncthreads();
                    for (int j = tid; j < n / 2; j += CSEL_THREADS) {
                        // pair j: the element with bit `stride` clear, and its partner
                        const int lo = ((j & ~(stride - 1)) << 1) | (j & (stride - 1)), hi = lo | stride;
                        const unsigned long long a = sk[lo], c = sk[hi];
                        if ((a > c) == ((lo & size) == 0)) {
                            sk[lo] = c;
                            sk[hi] = a;
                        }
                    }
                }
            __syncthreads();
            for (int j = tid; j < K; j += CSEL_THREADS) out[j] = (int32_t)(sk[j] & 0xffffu);
        } else {
            // more than CAND_BUF at or below the bound: the K smallest, one
            // at a time
            unsigned long long prev = 0ull;
            for (int r = 0; r < K; r++) {
                unsigned long long b = ~0ull;
                for (int i = tid; i < V; i += CSEL_THREADS) {
                    const float v = cand_logit(x, a1, a2, i);
                    if (v > -1e30f) {
                        const unsigned long long kk = cand_key(v, i);
                        if ((r == 0 || kk > prev) && kk < b) b = kk;
                    }
                }
#pragma unroll
                for (int o = 16; o; o >>= 1) b = umin64(b, __shfl_xor_sync(FULL, b, o));
                __syncthreads();
                if (lane == 0) sk[warp] = b;
                __syncthreads();
                b = sk[0];
                for (int w = 1; w < CSEL_THREADS / 32; w++) b = umin64(b, sk[w]);
                if (tid == 0) out[r] = (int32_t)(b & 0xffffu);
                prev = b;
            }
        }
    }
    for (int j = K + tid; j < k; j += CSEL_THREADS) out[j] = -1;
    if (tid == 0) {
        mo[s] = m;
        live_out[s] = live;
    }
}

// One warp per sequence (see above): lanes 0-3 add lane j's exps in order,
// 256 of each lane a chunk, while the warp's cp.async copies bring the next
// chunk into the other half of a shared double buffer. A row whose lane
// length is not a multiple of 256 is summed straight from global memory.
__global__ void __launch_bounds__(32) cand_sum_kernel(const float* ex, const float* logits, int V, const uint8_t* allow,
                                                      const float* mo, double* zo) {
    pdl_launch_dependents();
    pdl_wait();
    __shared__ __align__(16) float buf[2][4][256];
    const unsigned FULL = 0xffffffffu;
    const int s = blockIdx.x, lane = threadIdx.x;
    const int Q = V / 4;
    const float* er = ex + (size_t)s * 4 * Q;
    float acc = 0.f;
    if (Q % 256 == 0) {
        const int nchunk = Q / 256, seg = lane >> 3;
        auto fetch = [&](int c, int b) {
#pragma unroll
            for (int u = 0; u < 8; u++) {
                const int q4 = (lane & 7) + 8 * u;
                cp_async16(&buf[b][seg][4 * q4], er + (size_t)seg * Q + c * 256 + 4 * q4, true);
            }
            asm volatile("cp.async.commit_group;\n" ::);
        };
        fetch(0, 0);
        for (int c = 0; c < nchunk; c++) {
            if (c + 1 < nchunk) {
                fetch(c + 1, (c + 1) & 1);
                asm volatile("cp.async.wait_group 1;\n" ::);
            } else {
                asm volatile("cp.async.wait_group 0;\n" ::);
            }
            __syncwarp();
            if (lane < 4) {
                const float4* b4 = (const float4*)buf[c & 1][lane];
#pragma unroll 8
                for (int q = 0; q < 64; q++) {
                    const float4 e = b4[q];
                    acc = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(acc, e.x), e.y), e.z), e.w);
                }
            }
            __syncwarp();
        }
    } else if (lane < 4) {
        const float* el = er + (size_t)lane * Q;
        for (int i = 0; i < Q; i++) acc = __fadd_rn(acc, el[i]);
    }
    const float l1 = __shfl_sync(FULL, acc, 1), l2 = __shfl_sync(FULL, acc, 2), l3 = __shfl_sync(FULL, acc, 3);
    if (lane == 0) {
        const float m = mo[s];
        const float* x = logits + (size_t)s * V;
        const uint8_t* a1 = allow ? allow + (size_t)s * ((V + 7) / 8) : nullptr;
        double z = (double)__fadd_rn(__fadd_rn(acc, l1), __fadd_rn(l2, l3));
        for (int i = 4 * Q; i < V; i++) {
            const float v = cand_logit(x, a1, nullptr, i);
            if (v > -1e30f) z = __dadd_rn(z, exp(__dsub_rn((double)v, (double)m)));
        }
        zo[s] = z;
    }
}

cudaError_t launch_candidates(const float* logits, int S, int V, const uint8_t* allow, const uint8_t* allow_order, int k,
                              int32_t* ids, float* m, double* z, int32_t* live, float* ex, cudaStream_t st) {
    if (S < 1 || V < 1 || V > 65536 || k < 1 || k > CAND_MAXK) return cudaErrorInvalidValue;
    add_launches(2);
    launch_pdl(cand_select_kernel, dim3(S), dim3(CSEL_THREADS), 0, st, logits, V, allow, allow_order, k, ids, m, live, ex);
    launch_pdl(cand_sum_kernel, dim3(S), dim3(32), 0, st, (const float*)ex, logits, V, allow, (const float*)m, z);
    return cudaSuccess;
}

// ------------------------------------------------------------ probe heads

// infer.rs:1195-1211, 1707-1711: the lane mean (((x0 + x1) + x2) + x3) *
// 0.25 of each channel of row m = (s, i), at depth `depth` of position
// p0 + i. 192 threads, four channels each.
__global__ void record_cells_kernel(const float* xs, int T, int p0, int depth, int l1, int ncap, float* cells) {
    pdl_launch_dependents();
    pdl_wait();
    const int m = blockIdx.x, c4 = threadIdx.x;
    const int s = m / T, i = m % T;
    const float* x = xs + (size_t)m * 3072 + 4 * c4;
    const float4 a = *(const float4*)x, b = *(const float4*)(x + 768), c = *(const float4*)(x + 1536),
                 d = *(const float4*)(x + 2304);
    float4 o;
    o.x = __fmul_rn(__fadd_rn(__fadd_rn(__fadd_rn(a.x, b.x), c.x), d.x), 0.25f);
    o.y = __fmul_rn(__fadd_rn(__fadd_rn(__fadd_rn(a.y, b.y), c.y), d.y), 0.25f);
    o.z = __fmul_rn(__fadd_rn(__fadd_rn(__fadd_rn(a.z, b.z), c.z), d.z), 0.25f);
    o.w = __fmul_rn(__fadd_rn(__fadd_rn(__fadd_rn(a.w, b.w), c.w), d.w), 0.25f);
    *(float4*)(cells + (((size_t)s * ncap + p0 + i) * l1 + depth) * 768 + 4 * c4) = o;
}

void launch_record_cells(const float* xs, int S, int T, int p0, int depth, int l1, int ncap, float* cells, cudaStream_t st) {
    COUNT_LAUNCH();
    launch_pdl(record_cells_kernel, dim3(S * T), dim3(192), 0, st, xs, T, p0, depth, l1, ncap, cells);
}

// linalg.rs:262-277: the reference's own f32 exp (round half away, unfused).
__device__ __forceinline__ float fast_exp(float x) {
    x = fminf(fmaxf(x, -87.33654f), 88.72283f);
    const float k = roundf(__fmul_rn(x, 1.44269504088896340736f));
    const float r = __fsub_rn(__fsub_rn(x, __fmul_rn(k, 0.6933594f)), __fmul_rn(k, -2.1219444e-4f));
    float p = 1.9875691e-4f;
    p = __fadd_rn(__fmul_rn(p, r), 1.3981999e-3f);
    p = __fadd_rn(__fmul_rn(p, r), 8.333452e-3f);
    p = __fadd_rn(__fmul_rn(p, r), 4.1665796e-2f);
    p = __fadd_rn(__fmul_rn(p, r), 1.6666665e-1f);
    p = __fadd_rn(__fmul_rn(p, r), 5e-1f);
    const float y = __fadd_rn(__fadd_rn(__fmul_rn(__fmul_rn(p, r), r), r), 1.0f);
    return __fmul_rn(y, __uint_as_float((unsigned)((int)k + 127) << 23));
}

// linalg.rs:242-257 for n a multiple of 8, by the eight lanes 8g .. 8g + 7
// of a warp (lane j keeps accumulator j: x*y then +, in order), the total
// ((((a0 + a4) + (a1 + a5)) + (a2 + a6)) + (a3 + a7)) returned to all
// eight. Every lane of the warp takes part.
__device__ __forceinline__ float dot8_group(const float* a, const float* b, int n, int j) {
    float acc = 0.f;
    for (int c = 0; c < n / 8; c++) acc = __fadd_rn(acc, __fmul_rn(a[8 * c + j], b[8 * c + j]));
    const float t = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, 4, 8));  // lanes j < 4: a_j + a_(j+4)
    const float t0 = __shfl_sync(0xffffffffu, t, 0, 8), t1 = __shfl_sync(0xffffffffu, t, 1, 8);
    const float t2 = __shfl_sync(0xffffffffu, t, 2, 8), t3 = __shfl_sync(0xffffffffu, t, 3, 8);
    return __fadd_rn(__fadd_rn(__fadd_rn(t0, t1), t2), t3);
}

constexpr int HEAD_THREADS = 256;

// linalg.rs:309-323 over x[0..n) in shared memory, by the whole block:
// the max (order-free with FMAXNM), fast_exp(x - max) (0 for -inf), the
// sum in order by one thread, then x * (1 / sum).
__device__ void softmax_block(float* x, int n, float* red, float* s_val) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    float mx = -INFINITY;
    for (int i = tid; i < n; i += HEAD_THREADS) mx = fmaxnm(mx, x[i]);
#pragma unroll
    for (int o = 16; o; o >>= 1) mx = fmaxnm(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane == 0) red[warp] = mx;
    __syncthreads();
    float m = red[0];
    for (int w = 1; w < HEAD_THREADS / 32; w++) m = fmaxnm(m, red[w]);
    const bool none = m == -INFINITY;
    for (int i = tid; i < n; i += HEAD_THREADS) x[i] = (none || x[i] == -INFINITY) ? 0.f : fast_exp(__fsub_rn(x[i], m));
    __syncthreads();
    if (none) return;
    if (tid == 0) {
        float sum = 0.f;
        for (int i = 0; i < n; i++) sum = __fadd_rn(sum, x[i]);
        *s_val = __fdiv_rn(1.0f, sum);
    }
    __syncthreads();
    const float inv = *s_val;
    for (int i = tid; i < n; i += HEAD_THREADS) x[i] = __fmul_rn(x[i], inv);
    __syncthreads();
}

// heads.rs:21-43, one CTA per (sequence, depth-probe pair lk): scores of
// the T positions, softmax, the weighted sum of the cells in position
// order, rms_unit, times the gain.
__global__ void __launch_bounds__(HEAD_THREADS) probe_tokens_kernel(HeadW h, const float* cells, int T, int ncap, int l1,
                                                                    float inv, float* r) {
    pdl_launch_dependents();
    pdl_wait();
    extern __shared__ float sc[];  // [T]
    __shared__ float acc[768];
    __shared__ float red[HEAD_THREADS / 32];
    __shared__ float s_val;
    const int s = blockIdx.x, lk = blockIdx.y, l = lk / h.k, m = gridDim.y;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, g = lane >> 3, j = lane & 7;
    const float* probe = h.probes + (size_t)lk * 768;
    const float* base = cells + ((size_t)s * ncap * l1 + l) * 768;  // position t at + t * l1 * 768
    const size_t tstride = (size_t)l1 * 768;
    for (int tb = 0; tb < T; tb += 32) {
        const int t = tb + warp * 4 + g;
        const float v = dot8_group(base + (size_t)(t < T ? t : 0) * tstride, probe, 768, j);
        if (t < T && j == 0) sc[t] = __fmul_rn(v, inv);
    }
    __syncthreads();
    softmax_block(sc, T, red, &s_val);
    for (int c = tid; c < 768; c += HEAD_THREADS) {
        float a = 0.f;
        for (int t = 0; t < T; t++) a = __fadd_rn(a, __fmul_rn(sc[t], base[t * tstride + c]));
        acc[c] = a;
    }
    __syncthreads();
    if (tid == 0) {
        float ss = 0.f;
        for (int c = 0; c < 768; c++) ss = __fadd_rn(ss, __fmul_rn(acc[c], acc[c]));
        s_val = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, 768.0f), 1e-6f)));
    }
    __syncthreads();
    const float rr = s_val, gg = h.gain[lk];
    for (int c = tid; c < 768; c += HEAD_THREADS) r[((size_t)s * m + lk) * 768 + c] = __fmul_rn(__fmul_rn(acc[c], rr), gg);
}

// heads.rs:44-55, one CTA per (sequence, query): the m pooled rows'
// scores plus the row bias, softmax, the weighted sum of the rows in order.
__global__ void __launch_bounds__(HEAD_THREADS) probe_queries_kernel(HeadW h, const float* r, int m, float inv,
                                                                     float* pooled) {
    pdl_launch_dependents();
    pdl_wait();
    extern __shared__ float u[];  // [m]
    __shared__ float red[HEAD_THREADS / 32];
    __shared__ float s_val;
    const int s = blockIdx.x, qi = blockIdx.y;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, g = lane >> 3, j = lane & 7;
    const float* rs = r + (size_t)s * m * 768;
    const float* query = h.query + (size_t)qi * 768;
    for (int jb = 0; jb < m; jb += 32) {
        const int jj = jb + warp * 4 + g;
        const float v = dot8_group(rs + (size_t)(jj < m ? jj : 0) * 768, query, 768, j);
        if (jj < m && j == 0) u[jj] = __fadd_rn(__fmul_rn(v, inv), h.row_bias[(size_t)qi * m + jj]);
    }
    __syncthreads();
    softmax_block(u, m, red, &s_val);
    for (int c = tid; c < 768; c += HEAD_THREADS) {
        float a = 0.f;
        for (int jj = 0; jj < m; jj++) a = __fadd_rn(a, __fmul_rn(u[jj], rs[(size_t)jj * 768 + c]));
        pooled[((size_t)s * h.q + qi) * 768 + c] = a;
    }
}

// heads.rs:58-61, 68-90, one CTA per sequence: kind 0 the projection then
// unit norm, 1 the pool at unit norm, 2 the projection's first value.
__global__ void __launch_bounds__(HEAD_THREADS) probe_project_kernel(HeadW h, const float* pooled, int kind, float* out) {
    pdl_launch_dependents();
    pdl_wait();
    extern __shared__ float y[];  // [h.out]
    __shared__ float s_val;
    const int s = blockIdx.x, n = h.q * 768;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, g = lane >> 3, j = lane & 7;
    const float* pv = pooled + (size_t)s * n;
    if (kind == 1) {
        if (tid == 0) {
            float ss = 0.f;
            for (int c = 0; c < n; c++) ss = __fadd_rn(ss, __fmul_rn(pv[c], pv[c]));
            s_val = __fsqrt_rn(__fadd_rn(ss, 1e-12f));
        }
        __syncthreads();
        for (int c = tid; c < n; c += HEAD_THREADS) out[(size_t)s * n + c] = __fdiv_rn(pv[c], s_val);
        return;
    }
    for (int ob = 0; ob < h.out; ob += 32) {
        const int o = ob + warp * 4 + g;
        const float v = dot8_group(h.proj + (size_t)(o < h.out ? o : 0) * n, pv, n, j);
        if (o < h.out && j == 0) y[o] = __fadd_rn(v, h.bias[o]);
    }
    __syncthreads();
    if (kind == 2) {
        if (tid == 0) out[s] = y[0];
        return;
    }
    if (tid == 0) {
        float ss = 0.f;
        for (int o = 0; o < h.out; o++) ss = __fadd_rn(ss, __fmul_rn(y[o], y[o]));
        s_val = __fsqrt_rn(__fadd_rn(ss, 1e-12f));
    }
    __syncthreads();
    for (int o = tid; o < h.out; o += HEAD_THREADS) out[(size_t)s * h.out + o] = __fdiv_rn(y[o], s_val);
}

void launch_probe_head(HeadW h, const float* cells, int S, int T, int ncap, int l1, int kind, float* r, float* pooled,
                       float* out, cudaStream_t st) {
    // heads.rs:14: inv = 1 / (float)sqrt((double)d), divided in f32
    const float inv = 1.0f / (float)__builtin_sqrt(768.0);
    const int m = l1 * h.k;
    add_launches(3);
    launch_pdl(probe_tokens_kernel, dim3(S, m), dim3(HEAD_THREADS), (size_t)T * sizeof(float), st, h, cells, T, ncap, l1, inv, r);
    launch_pdl(probe_queries_kernel, dim3(S, h.q), dim3(HEAD_THREADS), (size_t)m * sizeof(float), st, h, (const float*)r, m, inv,
               pooled);
    launch_pdl(probe_project_kernel, dim3(S), dim3(HEAD_THREADS), (size_t)(h.out > 0 ? h.out : 1) * sizeof(float), st, h,
               (const float*)pooled, kind, out);
}

static cudaError_t init_attrs() {
    cudaFuncSetAttribute(attention_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)ATT_SMEM);
    cudaFuncSetAttribute(attention_kernel<5>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)ATT_SMEM);
    post_block_init();
    cudaFuncSetAttribute(post_row_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)POST_ROW_SMEM);
    cudaFuncSetAttribute(cq_mma_kernel<true, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)MMA_SMEM);
    cudaFuncSetAttribute(cq_mma_kernel<true, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)MMA_SMEM);
    cudaFuncSetAttribute(cq_mma_kernel<false, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)MMA_SMEM);
    return tc_prefill_init();
}

}  // namespace nd
