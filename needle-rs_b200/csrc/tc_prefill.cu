// The CQ/A8 matmul on the 5th-generation tensor cores, both combines.
//
// Prefill combine, qlinear.rs:353-363 (prefill_row_ref) with the
// block/remainder rule of qlinear.rs:395-419: for output row n and token m,
// each 128-wide group g gives an exact int32 sum s of int8 weight x int8
// activation products, and acc = fma(float(s), sc, acc) over g = 0..5 in
// order, sc = (norm * cbs) * sx for a sequence's first T/4*4 tokens and
// norm * (cbs * sx) for the rest.
//
// Decode combine, qlinear.rs:340-350 (decode_row_ref) for one-token rows:
// each group splits into four decode lanes (inputs p with (p % 32) / 8 ==
// l), lane l's int32 sum s_l feeds its own chain lanes[l] = fma(float(s_l),
// sc, lanes[l]) with sc = (sx * cbs) * norm, and the row is (l0 + l1) +
// (l2 + l3). In the engine's lane-major slot order decode lane l of a group
// is the 32 contiguous bytes l*32 .. l*32 + 31 (the 4-bit lane rule, which
// 3-bit records share; 2-bit records' split lanes stay on mma.sync).
//
// The integer sums come from tcgen05.mma.kind::i8 (A = 128 weight rows,
// B = the tile's tokens, K = 32 bytes an instruction, one per decode lane
// of a group) into s32 accumulators in tensor memory: the prefill combine
// chains a group's four MMAs into one accumulator (the group sum), the
// decode combine gives each its own (the lane sums), so the float chains
// see each sum exactly as the reference forms it. Each sum becomes a float
// by an integer add of the bit pattern of 1.5 * 2^23 and one exact f32
// subtraction instead of a quarter-rate int-to-float conversion. The
// operands arrive by TMA (cp.async.bulk.tensor, 128-byte swizzle) from this
// GPU's own HBM: the weights' int8 copy [out][768] and the A8 rows [M][768].
// No cluster multicast.
//
// One CTA per SM, persistent over a contiguous run of the output tiles
// (128 weight rows x 64 tokens for the prefill combine, x 32 tokens for
// the decode combine) in weight-tile-major order, warp-specialised: warp 0
// issues the TMA loads (a run's 128 weight rows stay resident in shared
// memory, all of K, one 96 KB box, reloaded only when the run reaches the
// next weight tile; each tile's activations, all of K, arrive as one 3-D
// box into a ring: the TMA cost here goes by loads more than by bytes, so
// few large boxes), warp 1 issues the MMAs into tensor-memory group
// buffers (all 512 columns), warp 18 writes each tile's column factors (per
// token and group: sx or cbs * sx) a tile ahead into a double buffer, and
// warps 2-17 read each group's sums back with tcgen05.ld (warp w reads
// lanes 32 (w % 4) .. + 31, i.e. 32 weight rows, and a quarter of the
// tile's token columns) and run the fma chains in registers, paired in
// f32x2; a tile's outputs are staged in shared memory and written by one
// TMA bulk store (when y's rows are 16-byte aligned; else by plain stores),
// which overlaps the next tile's work.
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

constexpr int TC_ROWS = 128;      // weight rows a tile (MMA M, tensor-memory lanes)
constexpr int TC_EPI_WARPS = 16;  // warps 2-17: 4 lane quarters x 4 column quarters
constexpr int TC_SCALE_WARP = 2 + TC_EPI_WARPS;
constexpr int TC_THREADS = 32 * (TC_SCALE_WARP + 1);  // + warp 0 TMA, warp 1 MMA, warp 18 column factors
constexpr uint32_t TC_TILE_BYTES = TC_ROWS * 128;     // one group of 128 weight rows: 16 KB
constexpr uint32_t TC_W_BYTES = 6 * TC_TILE_BYTES;    // a weight tile, all of K: 96 KB

// Per combine: tokens a tile (the MMA's N), the tensor-memory columns of a
// group's accumulators and how many group buffers fit the 512 columns, the
// activation ring depth (a stage is one tile's activations, all of K, one
// TMA box), and the kernel's shared memory.
template <bool DEC>
struct TcCfg {
    static constexpr int TOK = DEC ? 32 : 64;
    static constexpr int SLICE = DEC ? TOK : 0;         // columns between a group's lane accumulators
    static constexpr int GROUP_COLS = DEC ? 4 * TOK : TOK;
    static constexpr int BUFS = 512 / GROUP_COLS;
    // The MMA warp and the epilogue hand tensor memory over two groups at a
    // time (an acquire-ordered wait right after MMA issue costs ~300 cycles,
    // so per-group hand-offs would pace the pipeline): a slot is two group
    // buffers.
    static constexpr int SLOTS = BUFS / 2;
    static constexpr int CPT = TOK / 4;                  // token columns an epilogue thread reads
    static constexpr int STAGES = DEC ? 4 : 2;
    static constexpr uint32_t GRP_BYTES = TOK * 128;     // one group of the tile's tokens
    static constexpr uint32_t STAGE_BYTES = 6 * GRP_BYTES;
    static constexpr int OUT_HALVES = DEC ? 1 : 2;       // the output tile leaves in this many stores
    static constexpr uint32_t OUT_BYTES = TOK / OUT_HALVES * TC_ROWS * 4;
    static constexpr int NBARS = 2 * STAGES + 2 * BUFS + 6;
    static constexpr size_t SMEM = 1024 + TC_W_BYTES     // weight tile (1024-aligned)
                                   + (size_t)STAGES * STAGE_BYTES  // activation ring
                                   + OUT_BYTES                     // output staging [TOK / OUT_HALVES][128] f32
                                   + 2 * 6 * TOK * 4               // column factors [2][6][TOK]
                                   + 2 * TOK * 4                   // remainder flags [2][TOK]
                                   + NBARS * 8 + 16;               // barriers, tmem address, abort
    // kind::i8: s32 accumulator (c_format 2), signed A and B (formats 1),
    // both K-major, N = TOK (n_dim = N >> 3), M = 128 (m_dim = M >> 4)
    static constexpr uint32_t IDESC = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(TOK >> 3) << 17) | ((uint32_t)(TC_ROWS >> 4) << 24);
};
static_assert(TcCfg<false>::SMEM <= 227 * 1024 && TcCfg<true>::SMEM <= 227 * 1024, "shared memory per CTA");
static_assert(TcCfg<true>::SLOTS >= 2 && TcCfg<false>::SLOTS >= 2, "double-buffered slots of two group accumulators");
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

// A 2-D tiled TMA store of the f32 box {128 rows of y, the tile's tokens} from
// shared memory at (x = weight row, y = token); parts outside y's extents
// are not written.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, uint32_t src, int x, int y) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group [%0, {%2, %3}], [%1];\n" ::"l"((uint64_t)map),
                 "r"(src), "r"(x), "r"(y)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;\n" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;\n" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;\n" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory"); }
__device__ __forceinline__ void epi_sync() { asm volatile("bar.sync 1, %0;\n" ::"n"(TC_EPI_WARPS * 32) : "memory"); }

// A 3-D tiled TMA load of box {128 bytes, rows, 6 groups} at (0, y rows, 0):
// a tile's rows over all of K, laid out group after group, each group the
// [rows][128 bytes] tile the MMA descriptors address.
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, int y, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];\n" ::"r"(dst),
        "l"((uint64_t)map), "r"(0), "r"(y), "r"(0), "r"(bar)
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

__device__ __forceinline__ void mma_i8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrive on `bar` once every tcgen05 operation this thread issued so far has
// completed.
__device__ __forceinline__ void mma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory"); }

// 16 consecutive 32-bit columns of this warp's 32 lanes, and the wait for
// them (the registers tied to it, so no use is scheduled before it).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr)
        : "memory");
}
__device__ __forceinline__ void tmem_ld_wait16(uint32_t (&r)[16]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;\n"
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                   "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15])
                 :
                 : "memory");
}

// 8 consecutive 32-bit columns of this warp's 32 lanes.
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&r)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];\n"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr)
                 : "memory");
}

// Wait for this thread's tensor-memory loads, the four 8-column reads of a
// decode group tied to it.
__device__ __forceinline__ void tmem_ld_wait4x8(uint32_t (&r)[4][8]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;\n"
                 : "+r"(r[0][0]), "+r"(r[0][1]), "+r"(r[0][2]), "+r"(r[0][3]), "+r"(r[0][4]), "+r"(r[0][5]), "+r"(r[0][6]),
                   "+r"(r[0][7]), "+r"(r[1][0]), "+r"(r[1][1]), "+r"(r[1][2]), "+r"(r[1][3]), "+r"(r[1][4]), "+r"(r[1][5]),
                   "+r"(r[1][6]), "+r"(r[1][7]), "+r"(r[2][0]), "+r"(r[2][1]), "+r"(r[2][2]), "+r"(r[2][3]), "+r"(r[2][4]),
                   "+r"(r[2][5]), "+r"(r[2][6]), "+r"(r[2][7]), "+r"(r[3][0]), "+r"(r[3][1]), "+r"(r[3][2]), "+r"(r[3][3]),
                   "+r"(r[3][4]), "+r"(r[3][5]), "+r"(r[3][6]), "+r"(r[3][7])
                 :
                 : "memory");
}

// Every group sum s has |s| <= 128 * 128 * 128 < 2^22, so the int32 word
// s + bits(1.5 * 2^23) read as a float is 1.5 * 2^23 + s exactly, and one
// f32 subtraction gives float(s) without an int-to-float conversion. The
// accumulators start at bits(1.5 * 2^23) (written by the epilogue into every
// buffer before first use and again after reading it) and every MMA
// accumulates, so the words read back are already the biased floats.
constexpr uint32_t TC_MAGIC = 0x4B400000u;

// The bias into 4 / 8 / 16 consecutive 32-bit columns of this warp's 32 lanes
// (four columns a store: a store takes its columns' values in as many
// registers),
// and the wait for this thread's tensor-memory stores. (The stores touch
// tensor memory only; as volatile asm they stay ordered with the loads,
// waits and fences around them.)
__device__ __forceinline__ void tmem_bias4(uint32_t taddr) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1,%1,%1,%1};\n" ::"r"(taddr), "r"(TC_MAGIC));
}
__device__ __forceinline__ void tmem_bias8(uint32_t taddr) {
    tmem_bias4(taddr);
    tmem_bias4(taddr + 4);
}
__device__ __forceinline__ void tmem_bias16(uint32_t taddr) {
#pragma unroll
    for (int k = 0; k < 4; k++) tmem_bias4(taddr + 4 * k);
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory"); }

__device__ __forceinline__ float2 tc_sub2(float2 a, float2 b) {
    float2 d;
    asm("{\n.reg .b64 ra, rb, rd;\nmov.b64 ra, {%2, %3};\nmov.b64 rb, {%4, %5};\nsub.rn.f32x2 rd, ra, rb;\nmov.b64 {%0, %1}, rd;\n}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return d;
}

// Two independent IEEE products / fmas (sm_100 f32x2).
__device__ __forceinline__ float2 tc_mul2(float2 a, float2 b) {
    float2 d;
    asm("{\n.reg .b64 ra, rb, rd;\nmov.b64 ra, {%2, %3};\nmov.b64 rb, {%4, %5};\nmul.rn.f32x2 rd, ra, rb;\nmov.b64 {%0, %1}, rd;\n}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return d;
}
__device__ __forceinline__ float2 tc_fma2(float2 a, float2 b, float2 c) {
    float2 d;
    asm("{\n.reg .b64 ra, rb, rc, rd;\nmov.b64 ra, {%2, %3};\nmov.b64 rb, {%4, %5};\nmov.b64 rc, {%6, %7};\n"
        "fma.rn.f32x2 rd, ra, rb, rc;\nmov.b64 {%0, %1}, rd;\n}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
    return d;
}

__device__ __forceinline__ void pdl_wait_tc() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_tc() { asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory"); }

// ------------------------------------------------------------------ kernel

// DEC: the decode combine (one-token rows) instead of the prefill combine.
// REM (prefill only): some token rows are remainder rows (T % 4 != 0).
// BULK: the output tile leaves by a TMA store through map_y (y + col0 as
// [M][W.out] f32 rows ldy apart); else by plain stores.
template <bool DEC, bool REM, bool BULK>
__global__ void __launch_bounds__(TC_THREADS, 1)
    cq_tc_kernel(const __grid_constant__ CUtensorMap map_w, const __grid_constant__ CUtensorMap map_a,
                 const __grid_constant__ CUtensorMap map_y, DevMat W, const float* __restrict__ sx, int M, int T,
                 float* __restrict__ y, int ldy, int col0, int* err) {
    using C = TcCfg<DEC>;
    constexpr int TOK = C::TOK, STAGES = C::STAGES, CPT = C::CPT, BUFS = C::BUFS;
    pdl_launch_tc();
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t wtile = (raw + 1023u) & ~1023u;  // 1024-aligned for the 128-byte swizzle
    const uint32_t ring = wtile + TC_W_BYTES;
    uint8_t* gring = smem_raw + (ring - raw);
    float* stage_out = (float*)(gring + STAGES * C::STAGE_BYTES);  // [TOK / OUT_HALVES tokens][128 rows]
    float* colv = stage_out + TOK / C::OUT_HALVES * TC_ROWS;         // [2][6][TOK]
    int* remf = (int*)(colv + 2 * 6 * TOK);                         // [2][TOK]
    // full[STAGES] empty[STAGES] tfull[BUFS] tempty[BUFS] cfull[2] cempty[2] wfull wempty
    uint64_t* bars = (uint64_t*)(remf + 2 * TOK);
    uint32_t* tmem_slot = (uint32_t*)(bars + C::NBARS);
    volatile int* abort = (volatile int*)(tmem_slot + 1);
    const uint32_t bar0 = smem_u32(bars);
    auto full = [&](int s) { return bar0 + 8u * s; };
    auto empty = [&](int s) { return bar0 + 8u * (STAGES + s); };
    auto tfull = [&](int b) { return bar0 + 8u * (2 * STAGES + b); };
    auto tempty = [&](int b) { return bar0 + 8u * (2 * STAGES + BUFS + b); };
    auto cfull = [&](int t) { return bar0 + 8u * (2 * STAGES + 2 * BUFS + t); };
    auto cempty = [&](int t) { return bar0 + 8u * (2 * STAGES + 2 * BUFS + 2 + t); };
    const uint32_t wfull = bar0 + 8u * (2 * STAGES + 2 * BUFS + 4), wempty = wfull + 8u;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tilesN = (W.out + TC_ROWS - 1) / TC_ROWS, tilesM = (M + TOK - 1) / TOK;
    const int ntiles = tilesN * tilesM;
    // this CTA's run of tiles t0 .. t1 - 1; tile t is weight tile t / tilesM,
    // token tile t % tilesM
    const int t0 = (int)((long long)blockIdx.x * ntiles / gridDim.x), t1 = (int)((long long)(blockIdx.x + 1) * ntiles / gridDim.x);

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) {
            mbar_init(full(s), 1);
            mbar_init(empty(s), 1);
        }
        for (int b = 0; b < BUFS; b++) {
            mbar_init(tfull(b), 1);
            mbar_init(tempty(b), TC_EPI_WARPS);
        }
        for (int t = 0; t < 2; t++) {
            mbar_init(cfull(t), 1);
            mbar_init(cempty(t), TC_EPI_WARPS);
        }
        mbar_init(wfull, 1);
        mbar_init(wempty, 1);
        *abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
        tma_prefetch_map(&map_w);
        tma_prefetch_map(&map_a);
        if (BULK) tma_prefetch_map(&map_y);
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_u32(tmem_slot)),
                     "r"(512)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    // every accumulator buffer starts at the bias: epilogue warp e writes
    // its lane quarter and column quarter of each, before any MMA is issued
    if (warp >= 2 && warp < TC_SCALE_WARP) {
        const int q = warp & 3, c = (warp - 2) >> 2;
#pragma unroll 1
        for (int b = 0; b < C::BUFS; b++) {
            const uint32_t ta = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(b * C::GROUP_COLS + c * C::CPT);
            if constexpr (DEC) {
#pragma unroll
                for (int l = 0; l < 4; l++) tmem_bias8(ta + (uint32_t)(l * C::SLICE));
            } else {
                tmem_bias16(ta);
            }
        }
        tmem_st_wait();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();

    if (warp == 0) {
        // ---- TMA producer: lane 0 waits and issues, the warp stays converged;
        // one 3-D box a weight tile, one a tile's activations
        int it = 0, wk = 0, cur_n = -1;  // tiles, weight tiles loaded
        bool ok = true, waited = false;
        for (int t = t0; t < t1 && ok; t++, it++) {
            const int nt = t / tilesM, m0 = (t % tilesM) * TOK, s = it % STAGES;
            int good = 1;
            if (lane == 0) {
                if (nt != cur_n) {
                    // the previous weight tile must be done with (its last
                    // MMAs committed to wempty)
                    if (wk > 0) good = mbar_wait(wempty, (wk - 1) & 1, abort, err, 9);
                    if (good) {
                        mbar_expect_tx(wfull, TC_W_BYTES);
                        tma_load_3d(wtile, &map_w, nt * TC_ROWS, wfull);
                    }
                }
                if (good && it >= STAGES) good = mbar_wait(empty(s), ((it / STAGES) - 1) & 1, abort, err, 1);
                if (good) {
                    // the activations are the predecessor kernel's output
                    if (!waited) pdl_wait_tc();
                    mbar_expect_tx(full(s), C::STAGE_BYTES);
                    tma_load_3d(ring + s * C::STAGE_BYTES, &map_a, m0, full(s));
                }
            }
            waited = true;
            if (nt != cur_n) {
                cur_n = nt;
                wk++;
            }
            ok = __shfl_sync(0xffffffffu, good, 0) != 0;
        }
        if (lane == 0) {
            if (!waited) pdl_wait_tc();
            // drain: every load issued has landed before the CTA may exit
            for (int k = 0; k < STAGES && k < it; k++) {
                const int ik = it - 1 - k;
                mbar_wait(full(ik % STAGES), (ik / STAGES) & 1, abort, err, 5);
            }
            if (wk > 0) mbar_wait(wfull, (wk - 1) & 1, abort, err, 5);
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---- MMA issuer: lane 0 waits and issues, the warp stays converged
        int P = 0, it = 0, wk = 0, cur_n = -1;  // group pairs, tiles, weight tiles
        bool ok = true;
        for (int t = t0; t < t1 && ok; t++, it++) {
            const int nt = t / tilesM, s = it % STAGES;
            const bool last_of_w = t + 1 == t1 || (t + 1) / tilesM != nt;
            int good = 1;
            if (lane == 0) {
                if (nt != cur_n) good = mbar_wait(wfull, wk & 1, abort, err, 10);
                if (good) good = mbar_wait(full(s), (it / STAGES) & 1, abort, err, 2);
            }
            if (nt != cur_n) {
                cur_n = nt;
                wk++;
            }
            ok = __shfl_sync(0xffffffffu, good, 0) != 0;
            if (!ok) break;
            for (int pr = 0; pr < 3; pr++, P++) {
                const int sl = P % C::SLOTS;
                good = 1;
                if (lane == 0) {
                    if (P >= C::SLOTS) good = mbar_wait(tempty(sl), ((P / C::SLOTS) - 1) & 1, abort, err, 3);
                    if (good) {
                        tc_fence_after();
#pragma unroll
                        for (int h = 0; h < 2; h++) {
                            const int g = 2 * pr + h;
                            const uint32_t wa = wtile + g * TC_TILE_BYTES, aa = ring + s * C::STAGE_BYTES + g * C::GRP_BYTES;
                            const uint32_t d = tmem + (uint32_t)((2 * sl + h) * C::GROUP_COLS);
                            // K slice kk = decode lane kk of the group: the prefill
                            // combine sums the four into one accumulator, the decode
                            // combine keeps each in its own (TOK columns apart)
#pragma unroll
                            for (int kk = 0; kk < 4; kk++)
                                mma_i8(d + (uint32_t)(kk * C::SLICE), sw128_desc(wa + 32 * kk), sw128_desc(aa + 32 * kk), C::IDESC,
                                       1u);
                        }
                        mma_commit(tfull(sl));  // the two groups' sums are in slot sl
                        if (pr == 2) {
                            mma_commit(empty(s));                 // the tile's activations are read
                            if (last_of_w) mma_commit(wempty);    // the weight tile is done with
                        }
                    }
                }
                ok = __shfl_sync(0xffffffffu, good, 0) != 0;
                if (!ok) break;
            }
        }
        // every MMA issued has completed before the memory is freed
        if (lane == 0 && P > 0) {
            const int Pl = P - 1;
            mbar_wait(tfull(Pl % C::SLOTS), (Pl / C::SLOTS) & 1, abort, err, 6);
        }
        __syncwarp();
    } else if (warp == TC_SCALE_WARP) {
        // ---- column factors, a tile ahead, into buffer (tile count) % 2:
        // prefill, sx of each token and group for block rows and cbs * sx
        // for remainder rows (with the remainder flags); decode, sx * cbs
        // (0 past M)
        pdl_wait_tc();
        const float cbs = W.cbs;
        const int blocked = T / 4 * 4;
        int it = 0;
        bool ok = true;
        for (int tile = t0; tile < t1 && ok; tile++, it++) {
            const int m0 = (tile % tilesM) * TOK, tb = it & 1;
            int good = 1;
            if (lane == 0 && it >= 2) good = mbar_wait(cempty(tb), ((it >> 1) - 1) & 1, abort, err, 7);
            ok = __shfl_sync(0xffffffffu, good, 0) != 0;
            if (!ok) break;
            constexpr int PER = 6 * TOK / 32;  // factors a lane
            float v[PER];
#pragma unroll
            for (int k = 0; k < PER; k++) {
                const int i = lane + 32 * k, m = m0 + i / 6;  // sx is [M][6]: contiguous per tile
                v[k] = m < M ? __ldg(sx + (size_t)m0 * 6 + i) : 0.f;
                if (DEC) v[k] = __fmul_rn(v[k], cbs);
                else if ((m % T) >= blocked) v[k] = __fmul_rn(cbs, v[k]);
            }
            float* cv = colv + tb * 6 * TOK;
#pragma unroll
            for (int k = 0; k < PER; k++) {
                const int i = lane + 32 * k, j = i / 6, g = i % 6;
                cv[g * TOK + j] = v[k];
            }
            if (REM)
#pragma unroll
                for (int k = 0; k < TOK / 32; k++) {
                    const int j = lane + 32 * k;
                    remf[tb * TOK + j] = ((m0 + j) % T) >= blocked;
                }
            __syncwarp();
            if (lane == 0) mbar_arrive(cfull(tb));
        }
    } else {
        // ---- epilogue: warps 2-17; warp w reads lanes 32 (w % 4) .. + 31 (its
        // weight rows) and the column quarter c of the tile's tokens
        pdl_wait_tc();
        const int e = warp - 2, q = warp & 3, c = e >> 2;
        const bool leader = e == 0 && lane == 0;  // issues the tile's bulk store
        const float cbs = W.cbs;
        int P = 0, it = 0;  // group pairs, tiles
        bool ok = true;
        // the norms of this thread's weight row for the first tile; each tile
        // then loads the next tile's
        float nrm[6];
        {
            const int n = (t0 / tilesM) * TC_ROWS + q * 32 + lane;
#pragma unroll
            for (int g = 0; g < 6; g++) nrm[g] = (t0 < t1 && n < W.out) ? h2f(__ldg(W.norms + (size_t)n * 6 + g)) : 0.f;
        }
        for (int tile = t0; tile < t1; tile++, it++) {
            const int n0 = (tile / tilesM) * TC_ROWS, m0 = (tile % tilesM) * TOK, tb = it & 1;
            const int n = n0 + q * 32 + lane;  // this thread's weight row
            float nc[6];  // prefill: norm * cbs (block rows); remainder rows use norm alone
#pragma unroll
            for (int g = 0; g < 6; g++) nc[g] = __fmul_rn(nrm[g], cbs);
            float nrm_next[6];
            {
                const int t2 = tile + 1, n2 = (t2 / tilesM) * TC_ROWS + q * 32 + lane;
#pragma unroll
                for (int g = 0; g < 6; g++) nrm_next[g] = (t2 < t1 && n2 < W.out) ? h2f(__ldg(W.norms + (size_t)n2 * 6 + g)) : 0.f;
            }
            int good = 1;
            if (lane == 0 && ok) good = mbar_wait(cfull(tb), (it >> 1) & 1, abort, err, 8);
            ok = ok && __shfl_sync(0xffffffffu, good, 0) != 0;
            const float* cvt = colv + tb * 6 * TOK + c * CPT;
            const int* rf = remf + tb * TOK + c * CPT;
            const float2 mg = make_float2(12582912.0f, 12582912.0f);
            // prefill: acc[j] = the chain of tokens 2j, 2j + 1; decode: lanes[l][j]
            float2 acc[DEC ? 4 : 1][CPT / 2];
#pragma unroll
            for (int l = 0; l < (DEC ? 4 : 1); l++)
#pragma unroll
                for (int j = 0; j < CPT / 2; j++) acc[l][j] = make_float2(0.f, 0.f);
            for (int g = 0; g < 6; g++) {
                const int h = g & 1, sl = P % C::SLOTS, b = 2 * sl + h;
                if (h == 0) {
                    good = 1;
                    if (lane == 0 && ok) good = mbar_wait(tfull(sl), (P / C::SLOTS) & 1, abort, err, 4);
                    ok = ok && __shfl_sync(0xffffffffu, good, 0) != 0;
                    tc_fence_after();
                }
                const uint32_t ta = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(b * C::GROUP_COLS + c * CPT);
                const float* cv = cvt + g * TOK;
                // after the pair's second group is in registers, the slot is free
                auto release = [&]() {
                    if (h == 1) {
                        tmem_st_wait();  // the pair's buffers hold the bias again
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(tempty(sl));
                        P++;
                    }
                };
                if constexpr (DEC) {
                    uint32_t r[4][8];
                    if (ok) {
#pragma unroll
                        for (int l = 0; l < 4; l++) tmem_ld8(ta + (uint32_t)(l * C::SLICE), r[l]);
                        tmem_ld_wait4x8(r);
#pragma unroll
                        for (int l = 0; l < 4; l++) tmem_bias8(ta + (uint32_t)(l * C::SLICE));
                    } else {
#pragma unroll
                        for (int l = 0; l < 4; l++)
#pragma unroll
                            for (int j = 0; j < 8; j++) r[l][j] = 0u;
                    }
                    release();
                    const float2 nn = make_float2(nrm[g], nrm[g]);
#pragma unroll
                    for (int j = 0; j < 4; j++) {  // token pair (2j, 2j + 1)
                        // sc = (sx * cbs) * norm, shared by the four lanes
                        const float2 sc = tc_mul2(*(const float2*)(cv + 2 * j), nn);
#pragma unroll
                        for (int l = 0; l < 4; l++) {
                            const float2 s2 = tc_sub2(make_float2(__uint_as_float(r[l][2 * j]), __uint_as_float(r[l][2 * j + 1])), mg);
                            acc[l][j] = tc_fma2(s2, sc, acc[l][j]);
                        }
                    }
                } else {
                    uint32_t r[CPT];
                    if (ok) {
                        tmem_ld16(ta, r);
                        tmem_ld_wait16(r);
                        tmem_bias16(ta);
                    } else {
#pragma unroll
                        for (int j = 0; j < CPT; j++) r[j] = 0u;
                    }
                    release();
#pragma unroll
                    for (int j = 0; j < CPT / 2; j++) {  // token pair (2j, 2j + 1) of this quarter
                        const float2 s2 = tc_sub2(make_float2(__uint_as_float(r[2 * j]), __uint_as_float(r[2 * j + 1])), mg);
                        const float2 c2 = *(const float2*)(cv + 2 * j);
                        float2 f2 = make_float2(nc[g], nc[g]);
                        if (REM) {
                            if (rf[2 * j]) f2.x = nrm[g];
                            if (rf[2 * j + 1]) f2.y = nrm[g];
                        }
                        acc[0][j] = tc_fma2(s2, tc_mul2(f2, c2), acc[0][j]);
                    }
                }
            }
            // the column factors of this tile are read: free the buffer
            __syncwarp();
            if (lane == 0) mbar_arrive(cempty(tb));
            // the outputs of tokens 2j, 2j + 1: prefill, the chain; decode,
            // (l0 + l1) + (l2 + l3)
            float2 out[CPT / 2];
#pragma unroll
            for (int j = 0; j < CPT / 2; j++) {
                if constexpr (DEC) {
                    out[j].x = __fadd_rn(__fadd_rn(acc[0][j].x, acc[1][j].x), __fadd_rn(acc[2][j].x, acc[3][j].x));
                    out[j].y = __fadd_rn(__fadd_rn(acc[0][j].y, acc[1][j].y), __fadd_rn(acc[2][j].y, acc[3][j].y));
                } else {
                    out[j] = acc[0][j];
                }
            }
            if (BULK) {
                // stage the tile [token][row] (in OUT_HALVES rounds of token
                // quarters) and let one thread store each round; the previous
                // store must have read the staging first
                constexpr int QPH = 4 / C::OUT_HALVES;  // column quarters a round
#pragma unroll 1
                for (int hh = 0; hh < C::OUT_HALVES; hh++) {
                    if (leader) bulk_wait_read();
                    epi_sync();
                    if (c / QPH == hh) {
                        float* so = stage_out + ((c % QPH) * CPT) * TC_ROWS + q * 32 + lane;
#pragma unroll
                        for (int j = 0; j < CPT / 2; j++) {
                            so[(2 * j) * TC_ROWS] = out[j].x;
                            so[(2 * j + 1) * TC_ROWS] = out[j].y;
                        }
                        fence_async_smem();
                    }
                    epi_sync();
                    if (leader && ok) {
                        tma_store_2d(&map_y, smem_u32(stage_out), n0, m0 + hh * (TOK / C::OUT_HALVES));
                        bulk_commit();
                    }
                }
            } else if (ok && n < W.out) {
#pragma unroll
                for (int j = 0; j < CPT / 2; j++) {
                    const int m = m0 + c * CPT + 2 * j;
                    if (m < M) y[(size_t)m * ldy + col0 + n] = out[j].x;
                    if (m + 1 < M) y[(size_t)(m + 1) * ldy + col0 + n] = out[j].y;
                }
            }
#pragma unroll
            for (int g = 0; g < 6; g++) nrm[g] = nrm_next[g];
        }
        if (BULK && leader) bulk_wait_all();
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem), "r"(512) : "memory");
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

// The tensor map of an int8 [rows][768] matrix as 3-D boxes {128 bytes,
// box_rows rows, 6 groups} with the 128-byte swizzle: the groups (128 bytes
// apart in memory) are the outermost box dimension, so a box lands as six
// [box_rows][128 bytes] tiles, one per group. Rows past the end read as
// zeros.
static bool int8_rows_map(CUtensorMap* map, const void* base, int rows, int box_rows) {
    EncodeTiled enc = encode_fn();
    if (!enc || ((uintptr_t)base & 15) || rows < 1) return false;
    const cuuint64_t dims[3] = {128, (cuuint64_t)rows, 6};
    const cuuint64_t strides[2] = {768, 128};
    const cuuint32_t box[3] = {128, (cuuint32_t)box_rows, 6};
    const cuuint32_t estr[3] = {1, 1, 1};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// The tensor map of y + col0 as [M][out] f32 rows `ldy` floats apart, stored
// in boxes of 128 rows x box_tok tokens; false when the rows are not
// 16-byte aligned (the kernel then stores without TMA).
static bool f32_out_map(CUtensorMap* map, float* y, int col0, int out, int M, int ldy, int box_tok) {
    EncodeTiled enc = encode_fn();
    const float* base = y + col0;
    if (!enc || ((uintptr_t)base & 15) || ((size_t)ldy * 4) % 16 || out < 1 || M < 1) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)out, (cuuint64_t)M};
    const cuuint64_t strides[1] = {(cuuint64_t)ldy * 4};
    const cuuint32_t box[2] = {TC_ROWS, (cuuint32_t)box_tok};
    const cuuint32_t estr[2] = {1, 1};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
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
    cudaError_t e = cudaSuccess;
    auto set = [&](const void* f, size_t smem) {
        if (e == cudaSuccess) e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    };
    set((const void*)cq_tc_kernel<false, false, false>, TcCfg<false>::SMEM);
    set((const void*)cq_tc_kernel<false, false, true>, TcCfg<false>::SMEM);
    set((const void*)cq_tc_kernel<false, true, false>, TcCfg<false>::SMEM);
    set((const void*)cq_tc_kernel<false, true, true>, TcCfg<false>::SMEM);
    set((const void*)cq_tc_kernel<true, false, false>, TcCfg<true>::SMEM);
    set((const void*)cq_tc_kernel<true, false, true>, TcCfg<true>::SMEM);
    // the error word's address, looked up now (before any stream capture)
    if (e == cudaSuccess && !tc_err_ptr()) e = cudaErrorInvalidSymbol;
    return e;
}

template <bool DEC>
static cudaError_t launch_tc(DevMat W, const int8_t* act, const float* sx, int M, int T, float* y, int ldy, int col0,
                             cudaStream_t st) {
    using C = TcCfg<DEC>;
    int* err = tc_err_ptr();
    if (!W.w8 || W.in_dim != 768 || W.groups != 6 || M < 1 || !err) return cudaErrorInvalidValue;
    CUtensorMap mw, ma, my;
    if (!int8_rows_map(&mw, W.w8, W.out, TC_ROWS) || !int8_rows_map(&ma, act, M, C::TOK)) return cudaErrorInvalidValue;
    const bool bulk = f32_out_map(&my, y, col0, W.out, M, ldy, C::TOK / C::OUT_HALVES);
    if (!bulk) my = mw;  // unused by the plain-store variant
    const int ntiles = ((W.out + TC_ROWS - 1) / TC_ROWS) * ((M + C::TOK - 1) / C::TOK);
    const int grid = std::min(ntiles, sm_count_tc());
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(TC_THREADS);
    cfg.dynamicSmemBytes = C::SMEM;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = st ? 1 : 0;
    if (DEC) {
        if (bulk) return cudaLaunchKernelEx(&cfg, cq_tc_kernel<true, false, true>, mw, ma, my, W, sx, M, T, y, ldy, col0, err);
        return cudaLaunchKernelEx(&cfg, cq_tc_kernel<true, false, false>, mw, ma, my, W, sx, M, T, y, ldy, col0, err);
    }
    const bool rem = T % 4 != 0;
    if (rem && bulk) return cudaLaunchKernelEx(&cfg, cq_tc_kernel<false, true, true>, mw, ma, my, W, sx, M, T, y, ldy, col0, err);
    if (rem) return cudaLaunchKernelEx(&cfg, cq_tc_kernel<false, true, false>, mw, ma, my, W, sx, M, T, y, ldy, col0, err);
    if (bulk) return cudaLaunchKernelEx(&cfg, cq_tc_kernel<false, false, true>, mw, ma, my, W, sx, M, T, y, ldy, col0, err);
    return cudaLaunchKernelEx(&cfg, cq_tc_kernel<false, false, false>, mw, ma, my, W, sx, M, T, y, ldy, col0, err);
}

cudaError_t launch_cq_prefill_tc(DevMat W, const int8_t* act, const float* sx, int M, int T, float* y, int ldy, int col0,
                                 cudaStream_t st) {
    if (T < 2) return cudaErrorInvalidValue;
    return launch_tc<false>(W, act, sx, M, T, y, ldy, col0, st);
}

cudaError_t launch_cq_decode_tc(DevMat W, const int8_t* act, const float* sx, int M, float* y, int ldy, int col0,
                                cudaStream_t st) {
    if (W.width == 2) return cudaErrorInvalidValue;  // the 2-bit lane rule splits a lane's 32 bytes
    return launch_tc<true>(W, act, sx, M, 1, y, ldy, col0, st);
}

}  // namespace nd
