// The CQ/A8 matmul's prefill combine on the 5th-generation tensor cores.
//
// qlinear.rs:353-363 (prefill_row_ref) with the block/remainder rule of
// qlinear.rs:395-419: for output row n and token m, each 128-wide group g
// gives an exact int32 sum s of int8 weight x int8 activation products, and
// acc = fma(float(s), sc, acc) over g = 0..5 in order, sc = (norm * cbs) * sx
// for a sequence's first T/4*4 tokens and norm * (cbs * sx) for the rest.
//
// The integer sums come from tcgen05.mma.kind::i8 (A = 128 weight rows,
// B = 128 tokens, K = 32 bytes an instruction, four per group) into an s32
// accumulator in tensor memory: one 128 x 128 accumulator per group, so the
// float chain sees each group's sum exactly as the reference forms it. The
// operands arrive by TMA (cp.async.bulk.tensor, 128-byte swizzle) from this
// GPU's own HBM: the weights' int8 copy [out][768] and the A8 rows [M][768]
// (both in the engine's lane-major slot order within a group, which a full
// group sum does not see). No cluster multicast.
//
// One CTA per SM, persistent over 128 x 128 output tiles, warp-specialised:
// warp 0 issues the TMA loads into a 4-stage ring, warp 1 issues the MMAs
// into 4 tensor-memory buffers of 128 columns, warps 2-9 read each group's
// sums back with tcgen05.ld (warp w reads lanes 32 (w % 4) .. + 31, i.e. 32
// weight rows, and half of the 128 token columns) and run the fma chains in
// registers; the tile's outputs leave as coalesced 128-byte rows of y.
//
// Every wait on an mbarrier is bounded: on expiry the kernel records an
// error code in *err, every role stops issuing work, waits (bounded) for
// the copies and MMAs it has in flight, and the tensor memory is freed.

#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>
#include <mutex>
#include <stdexcept>
#include <string>

#include "kernels.h"
#include "numerics.cuh"

namespace nd {

constexpr int TC_ROWS = 128;     // weight rows a tile (MMA M, tensor-memory lanes)
constexpr int TC_TOK = 128;      // tokens a tile (MMA N, tensor-memory columns)
constexpr int TC_STAGES = 4;     // shared-memory ring of (weights, activations) group tiles
constexpr int TC_BUFS = 4;       // tensor-memory accumulators of 128 columns (all 512)
constexpr int TC_THREADS = 320;  // warp 0 TMA, warp 1 MMA, warps 2-9 epilogue
constexpr int TC_EPI_WARPS = 8;
constexpr uint32_t TC_TILE_BYTES = TC_ROWS * 128;                   // one group of 128 rows: 16 KB
constexpr uint32_t TC_STAGE_BYTES = 2 * TC_TILE_BYTES;              // weights + activations
constexpr size_t TC_SMEM = 1024 + (size_t)TC_STAGES * TC_STAGE_BYTES  // ring (1024-aligned)
                           + 6 * TC_TOK * 4                           // column factors [6][128]
                           + TC_TOK * 4                               // remainder flags
                           + 16 * 8 + 16;                             // barriers, tmem address, abort
constexpr uint32_t TC_SPIN = 1u << 20;  // try_wait rounds before a wait counts as failed

// --------------------------------------------------------------- PTX helpers

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n.reg .pred p;\nmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\nselp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// Wait for phase `parity` of a barrier, giving up after TC_SPIN rounds or
// once another role has given up (*abort set): false then, with the code
// recorded once in *err.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort, int* err, int code) {
    for (uint32_t it = 0; it < TC_SPIN; it++) {
        if (mbar_try(bar, parity)) return true;
        if ((it & 255) == 255 && *abort) return false;
    }
    *abort = 1;
    atomicCAS(err, 0, code);
    return false;
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(bar), "r"(bytes) : "memory");
}

// A 2-D tiled TMA load of box {128 bytes, 128 rows} at (x bytes, y rows),
// completing `bar`'s transaction count. x is a multiple of 128.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];\n" ::"r"(dst),
        "l"((uint64_t)map), "r"(x), "r"(y), "r"(bar)
        : "memory");
}

__device__ __forceinline__ void tma_prefetch_map(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];\n" ::"l"((uint64_t)map) : "memory");
}

// Shared-memory matrix descriptor of tcgen05 for a K-major operand in the
// 128-byte swizzle TMA writes: rows of 128 bytes, 8-row atoms 1024 bytes
// apart (stride byte offset), version 1, layout SWIZZLE_128B (2).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) | ((uint64_t)1 << 46) |
           ((uint64_t)2 << 61);
}

// Instruction descriptor, kind::i8: s32 accumulator (c_format 2), signed A
// and B (formats 1), both K-major, N = 128 (n_dim = N >> 3), M = 128
// (m_dim = M >> 4).
constexpr uint32_t TC_IDESC = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(TC_TOK >> 3) << 17) | ((uint32_t)(TC_ROWS >> 4) << 24);

__device__ __forceinline__ void mma_i8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
    asm volatile(
        "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(TC_IDESC), "r"(accumulate)
        : "memory");
}

// Arrive on `bar` once every tcgen05 operation this thread issued so far has
// completed.
__device__ __forceinline__ void mma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory"); }

// 32 consecutive 32-bit columns of this warp's 32 lanes.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,"
        "%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
          "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr)
        : "memory");
}

__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory"); }

__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, %0;\n" ::"n"(TC_EPI_WARPS * 32) : "memory"); }

__device__ __forceinline__ void pdl_wait_tc() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_tc() { asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory"); }

// ------------------------------------------------------------------ kernel

// REM: some token rows are remainder rows (T % 4 != 0).
template <bool REM>
__global__ void __launch_bounds__(TC_THREADS, 1)
    cq_tc_prefill_kernel(const __grid_constant__ CUtensorMap map_w, const __grid_constant__ CUtensorMap map_a, DevMat W,
                         const float* __restrict__ sx, int M, int T, float* __restrict__ y, int ldy, int col0, int* err) {
    pdl_launch_tc();
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t ring = (raw + 1023u) & ~1023u;  // 1024-aligned for the 128-byte swizzle
    uint8_t* gring = smem_raw + (ring - raw);
    float* colv = (float*)(gring + TC_STAGES * TC_STAGE_BYTES);  // [6][128]
    int* remf = (int*)(colv + 6 * TC_TOK);                       // [128]
    uint64_t* bars = (uint64_t*)(remf + TC_TOK);                 // full[4] empty[4] tfull[4] tempty[4]
    uint32_t* tmem_slot = (uint32_t*)(bars + 16);
    volatile int* abort = (volatile int*)(tmem_slot + 1);
    const uint32_t bar0 = smem_u32(bars);
    auto full = [&](int s) { return bar0 + 8u * s; };
    auto empty = [&](int s) { return bar0 + 8u * (4 + s); };
    auto tfull = [&](int b) { return bar0 + 8u * (8 + b); };
    auto tempty = [&](int b) { return bar0 + 8u * (12 + b); };

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tilesN = (W.out + TC_ROWS - 1) / TC_ROWS, tilesM = (M + TC_TOK - 1) / TC_TOK;
    const int ntiles = tilesN * tilesM;

    if (threadIdx.x == 0) {
        for (int s = 0; s < TC_STAGES; s++) {
            mbar_init(full(s), 1);
            mbar_init(empty(s), 1);
        }
        for (int b = 0; b < TC_BUFS; b++) {
            mbar_init(tfull(b), 1);
            mbar_init(tempty(b), TC_EPI_WARPS);
        }
        *abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
        tma_prefetch_map(&map_w);
        tma_prefetch_map(&map_a);
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_u32(tmem_slot)),
                     "r"(TC_BUFS * TC_TOK)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ---- TMA producer: lane 0 waits and issues, the warp stays converged
        int G = 0;  // group counter across this CTA's tiles
        bool ok = true, waited = false;
        for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x) {
            const int n0 = (tile % tilesN) * TC_ROWS, m0 = (tile / tilesN) * TC_TOK;
            for (int g = 0; g < 6; g++, G++) {
                const int s = G % TC_STAGES;
                int good = 1;
                if (lane == 0) {
                    if (G >= TC_STAGES) good = mbar_wait(empty(s), ((G / TC_STAGES) - 1) & 1, abort, err, 1);
                    if (good) {
                        const uint32_t dst = ring + s * TC_STAGE_BYTES;
                        mbar_expect_tx(full(s), TC_STAGE_BYTES);
                        tma_load_2d(dst, &map_w, g * 128, n0, full(s));
                        // the activations are the predecessor kernel's output
                        if (!waited) pdl_wait_tc();
                        tma_load_2d(dst + TC_TILE_BYTES, &map_a, g * 128, m0, full(s));
                    }
                }
                waited = true;
                ok = __shfl_sync(0xffffffffu, good, 0) != 0;
                if (!ok) break;
            }
        }
        if (lane == 0) {
            if (!waited) pdl_wait_tc();
            // drain: every load issued has landed before the CTA may exit
            for (int k = 0; k < TC_STAGES && k < G; k++) {
                const int Gk = G - 1 - k, s = Gk % TC_STAGES;
                mbar_wait(full(s), (Gk / TC_STAGES) & 1, abort, err, 5);
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---- MMA issuer: lane 0 waits and issues, the warp stays converged
        int G = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x) {
            for (int g = 0; g < 6; g++, G++) {
                const int s = G % TC_STAGES, b = G % TC_BUFS;
                int good = 1;
                if (lane == 0) {
                    good = mbar_wait(full(s), (G / TC_STAGES) & 1, abort, err, 2);
                    if (good && G >= TC_BUFS) good = mbar_wait(tempty(b), ((G / TC_BUFS) - 1) & 1, abort, err, 3);
                    if (good) {
                        tc_fence_after();
                        const uint32_t wa = ring + s * TC_STAGE_BYTES, aa = wa + TC_TILE_BYTES;
                        const uint32_t d = tmem + (uint32_t)(b * TC_TOK);
#pragma unroll
                        for (int kk = 0; kk < 4; kk++) mma_i8(d, sw128_desc(wa + 32 * kk), sw128_desc(aa + 32 * kk), kk);
                        mma_commit(empty(s));  // the stage is free once these MMAs have read it
                        mma_commit(tfull(b));  // the group's sums are in buffer b
                    }
                }
                ok = __shfl_sync(0xffffffffu, good, 0) != 0;
                if (!ok) break;
            }
        }
        // every MMA issued has completed before the memory is freed
        if (lane == 0 && G > 0) {
            const int Gl = G - 1;
            mbar_wait(tfull(Gl % TC_BUFS), (Gl / TC_BUFS) & 1, abort, err, 6);
        }
        __syncwarp();
    } else {
        // ---- epilogue: warps 2-9
        pdl_wait_tc();
        const int e = warp - 2, q = warp & 3, half = e >> 2;
        const int et = threadIdx.x - 64;  // 0..255
        const float cbs = W.cbs;
        const int blocked = T / 4 * 4;
        int G = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
            const int n0 = (tile % tilesN) * TC_ROWS, m0 = (tile / tilesN) * TC_TOK;
            const int n = n0 + q * 32 + lane;  // this thread's weight row
            // the tile's column factors: sx (block rows) or cbs * sx
            // (remainder rows) of each token and group
            epi_bar();
            for (int i = et; i < 6 * TC_TOK; i += TC_EPI_WARPS * 32) {
                const int g = i / TC_TOK, j = i % TC_TOK, m = m0 + j;
                float v = 0.f;
                if (m < M) {
                    const float s = __ldg(sx + (size_t)m * 6 + g);
                    v = (m % T) < blocked ? s : __fmul_rn(cbs, s);
                }
                colv[g * TC_TOK + j] = v;
            }
            if (REM)
                for (int j = et; j < TC_TOK; j += TC_EPI_WARPS * 32) remf[j] = ((m0 + j) % T) >= blocked;
            // the row factors: norm * cbs (block rows), norm (remainder rows)
            float nrm[6], nc[6];
#pragma unroll
            for (int g = 0; g < 6; g++) {
                nrm[g] = n < W.out ? h2f(__ldg(W.norms + (size_t)n * 6 + g)) : 0.f;
                nc[g] = __fmul_rn(nrm[g], cbs);
            }
            epi_bar();
            float acc[64];
#pragma unroll
            for (int j = 0; j < 64; j++) acc[j] = 0.f;
            for (int g = 0; g < 6; g++, G++) {
                const int b = G % TC_BUFS;
                if (ok) ok = mbar_wait(tfull(b), (G / TC_BUFS) & 1, abort, err, 4);
                tc_fence_after();
                uint32_t r0[32], r1[32];
                const uint32_t ta = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(b * TC_TOK + half * 64);
                if (ok) {
                    tmem_ld32(ta, r0);
                    tmem_ld32(ta + 32, r1);
                    tmem_ld_wait();
                } else {
#pragma unroll
                    for (int j = 0; j < 32; j++) r0[j] = r1[j] = 0u;
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(tempty(b));
                const float* cv = colv + g * TC_TOK + half * 64;
#pragma unroll
                for (int j = 0; j < 64; j++) {
                    const float s = (float)(int)(j < 32 ? r0[j] : r1[j - 32]);
                    float f = nc[g];
                    if (REM && remf[half * 64 + j]) f = nrm[g];
                    acc[j] = __fmaf_rn(s, __fmul_rn(f, cv[j]), acc[j]);
                }
            }
            if (ok && n < W.out) {
#pragma unroll
                for (int j = 0; j < 64; j++) {
                    const int m = m0 + half * 64 + j;
                    if (m < M) y[(size_t)m * ldy + col0 + n] = acc[j];
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem), "r"(TC_BUFS * TC_TOK) : "memory");
    }
}

// ------------------------------------------------------------------- host

typedef CUresult (*EncodeTiled)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*, const cuuint64_t*,
                                const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiled encode_fn() {
    static EncodeTiled fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (EncodeTiled)p;
    });
    return fn;
}

// The tensor map of an int8 [rows][768] matrix read in boxes of 128 bytes x
// 128 rows with the 128-byte swizzle; rows past the end read as zeros.
static bool int8_rows_map(CUtensorMap* map, const void* base, int rows) {
    EncodeTiled enc = encode_fn();
    if (!enc || ((uintptr_t)base & 15) || rows < 1) return false;
    const cuuint64_t dims[2] = {768, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {768};
    const cuuint32_t box[2] = {128, 128};
    const cuuint32_t estr[2] = {1, 1};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

static int sm_count_tc() {
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

// The error word of the bounded waits, one per device (a module variable,
// so no allocation); 0 = no wait has expired.
static __device__ int g_tc_err;

static int* tc_err_ptr() {
    static std::atomic<int*> ptrs[64];
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return nullptr;
    int* p = ptrs[dev].load(std::memory_order_acquire);
    if (!p) {
        void* q = nullptr;
        if (cudaGetSymbolAddress(&q, g_tc_err) != cudaSuccess) return nullptr;
        p = (int*)q;
        ptrs[dev].store(p, std::memory_order_release);
    }
    return p;
}

int tc_prefill_error() {
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_tc_err, sizeof(int)) != cudaSuccess) return -1;
    if (v) {
        const int zero = 0;
        cudaMemcpyToSymbol(g_tc_err, &zero, sizeof(int));
    }
    return v;
}

cudaError_t tc_prefill_init() {
    cudaError_t e = cudaFuncSetAttribute(cq_tc_prefill_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)TC_SMEM);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(cq_tc_prefill_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)TC_SMEM);
    return e;
}

cudaError_t launch_cq_prefill_tc(DevMat W, const int8_t* act, const float* sx, int M, int T, float* y, int ldy, int col0,
                                 cudaStream_t st) {
    int* err = tc_err_ptr();
    if (!W.w8 || W.in_dim != 768 || W.groups != 6 || M < 1 || T < 2 || !err) return cudaErrorInvalidValue;
    CUtensorMap mw, ma;
    if (!int8_rows_map(&mw, W.w8, W.out) || !int8_rows_map(&ma, act, M)) return cudaErrorInvalidValue;
    const int ntiles = ((W.out + TC_ROWS - 1) / TC_ROWS) * ((M + TC_TOK - 1) / TC_TOK);
    const int grid = std::min(ntiles, sm_count_tc());
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(TC_THREADS);
    cfg.dynamicSmemBytes = TC_SMEM;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = st ? 1 : 0;
    if (T % 4)
        return cudaLaunchKernelEx(&cfg, cq_tc_prefill_kernel<true>, mw, ma, W, sx, M, T, y, ldy, col0, err);
    return cudaLaunchKernelEx(&cfg, cq_tc_prefill_kernel<false>, mw, ma, W, sx, M, T, y, ldy, col0, err);
}

}  // namespace nd
