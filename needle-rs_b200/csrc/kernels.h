// Kernel launchers of the Needle 3 packed forward pass on sm_100a.
//
// Row index m of a step is (sequence s, token i) = (m / T, m % T): every
// sequence of a batch feeds the same T tokens at the same positions
// p0 .. p0 + T - 1. Caches are per sequence and per layer.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace nd {

// A CQ matrix as the archive stores it: codes [out][groups][16 * width]
// (LSB-first, 8 codes per `width` bytes), f16 group norms [out][groups],
// and its codebook (qlinear.rs:43-61, 244-265). A fused projection whose
// parts differ in codebook is several DevMats, one per run of equal parts.
struct DevMat {
    const uint8_t* codes = nullptr;
    const uint16_t* norms = nullptr;
    int out = 0, in_dim = 0, groups = 0;
    // Bits per code in memory: 2 (2-bit and ternary records), 3 or 4. Width
    // 2 splits a group into decode lanes by (p % 64) / 16, the others by
    // (p % 32) / 8 (qlinear.rs:333).
    int width = 4;
    float cbs = 1.0f;       // scale of the int8 codebook
    uint32_t vals4[4] = {0, 0, 0, 0};  // code -> int8 codebook value (16 bytes)
    float fvals[16] = {};   // code -> f32 codebook value (row dequant)
    // The same codes expanded through the int8 codebook, [out][groups*128],
    // each group lane-major (lane_major_pos in kernels.cu): the operand the
    // tensor-core kernel streams when many rows share a step.
    const int8_t* w8 = nullptr;
};

// Row stride (floats) of the conditioning weights and of the conditioning
// input as the post block keeps them: chain (set, k) of cond_weights reads
// element set + 4 n at column n, so a chain's operands are 16-byte runs;
// 192 columns padded to 196 so the eight chains of a quarter-warp start in
// distinct bank quads.
constexpr int COND_LD = 196;

// One layer's weights on the device (small weights widened to f32, which
// is exact for the archive's f16 values).
struct LayerW {
    const float *norm_in, *q_taps, *k_taps, *v_taps, *q_norm, *k_norm, *post_norm, *pre_hada;
    const float *d1, *d2, *b2, *d3, *d4, *kron[6], *cond_u;
    const float* cond_v;  // [32][COND_LD]: row 8 set + k, column n = cond_v[set + 4 n][k]
    const int8_t* phi_q;  // [24][3072]
    const float* phi_s;   // [24]
    float attn_gate, a_pre, a_post, a_res;
    float b_pre[4], b_post[4], b_res[16];
};

// A probe-pooling head (weights.rs:60-76) on the device, dequantized to f32:
// probes [(L+1) * k][d], gain [(L+1) * k], query [q][d], row_bias
// [q][(L+1) * k], proj [out][q * d], bias [out].
struct HeadW {
    int k = 0, q = 0, out = 0;
    const float *probes = nullptr, *gain = nullptr, *query = nullptr, *row_bias = nullptr, *proj = nullptr,
                *bias = nullptr;
};

// Per-sequence caches of one batch.
struct Caches {
    int S, L, cap;        // sequences, layers, KV slots per sequence
    int vgroups;          // value groups per sequence and head: ceil(cap / 4)
    int8_t* k8;           // [S][L][2][cap][48]
    float* ks;            // [S][L][2][cap]
    int8_t* v8;           // [S][L][2][vgroups][64][4]: position 4g + j's byte j of a dimension word
    float* vs;            // [S][L][2][cap]
    float* hist;          // [S][L][HIST_RING][800] pre-tap q|k|v rows by position
    int8_t* ev8;          // [S][sites][ENG_RING][768] engram value history
    float* evs;           // [S][sites][ENG_RING][24]
    int32_t* tokens;      // [S][cap]
    // positions every sequence has been fed before this step, on the device:
    // kernels read their positions here, so a captured step replays anywhere
    const int32_t* len;
};

// Pre-tap rows kept per (sequence, layer), by position modulo the ring: the
// conv reads two back, and each row writes its own row in the same kernel,
// so a chunk's 32 new positions must not reuse the two slots rows 0 and 1
// read (32 + 2); it is also the reference's rollback depth plus the taps
// (ROLLBACK = 32, model.rs:184; keep = taps - 1 + ROLLBACK, infer.rs:1489).
constexpr int HIST_RING = 34;
// Engram value history kept per (sequence, site), by position: a chunk's 32
// rows are all written before the dilated conv reads 3 taps of dilation 3
// back, so the ring must hold 32 + 9 positions.
constexpr int ENG_RING = 64;
// RoPE rows kept by position (state of launch_rope_rows): a one-token step
// continues the newest row by the angle-addition recurrence, and after a
// rollback of up to 32 positions the row before the new end must still be
// there (the reference keeps ROLLBACK + 1 rows, infer.rs:1735-1742).
constexpr int ROPE_RING = 33;
// The longest key list the attention kernel takes: 32 key chunks of 256.
constexpr int ATT_MAX_KEYS = 8192;

// The current device's SM count (looked up once per device).
int device_sm_count();
// Kernels this process has launched through the launchers below.
long long launch_count();
// Kernels a replayed CUDA graph launched (counted with the others).
void add_launches(long long n);

// The Hadamard scale (float)(1/sqrt(128)) and kernel attributes, once per
// device before its first launch.
void set_constants(float hs128);
// Slot of input p (< 128) of a group in the lane-major A8 / w8 layout.
int lane_major_slot(int p);

void launch_write_tokens(const int32_t* ids, int S, int T, int p0, Caches c, cudaStream_t st);
void launch_embed(DevMat emb, const int32_t* ids, int M, float* xs, cudaStream_t st);
void launch_prep_act(const float* x, int ldx, int K, int M, int8_t* act, float* sx, cudaStream_t st);
// y[m][col0 + n] for n < W.out. T sets the combine per row: T == 1 the
// decode combine (the code-reading GEMV for up to 4 rows, int8 mma.sync tiles
// up to 63, the tcgen05 kernel from 64, 2-bit matrices on mma.sync), else the
// prefill combine with the block/remainder rule over each sequence's T rows
// (mma.sync below 256 rows, tcgen05 from 256). cudaErrorInvalidValue (nothing
// launched) unless W reads 768 inputs and carries its w8 copy.
cudaError_t launch_cq_gemm(DevMat W, const int8_t* act, const float* sx, int M, int T, float* y, int ldy, int col0,
                           cudaStream_t st);
// The prefill combine (T > 1) on tcgen05 tensor cores fed by TMA (tc_prefill.cu);
// launch_cq_gemm routes T > 1 here. tc_prefill_init sets its kernel
// attributes on the current device; tc_prefill_error returns (and clears)
// the current device's error word: nonzero when a bounded wait of the
// kernel expired (read it after synchronising the stream).
cudaError_t launch_cq_prefill_tc(DevMat W, const int8_t* act, const float* sx, int M, int T, float* y, int ldy, int col0,
                                 cudaStream_t st);
// The decode combine on the same tensor-core kernel (launch_cq_gemm routes
// batched one-token steps here); not for 2-bit matrices, whose decode lanes
// are split runs of the group.
cudaError_t launch_cq_decode_tc(DevMat W, const int8_t* act, const float* sx, int M, float* y, int ldy, int col0,
                                cudaStream_t st);
cudaError_t tc_prefill_init();
int tc_prefill_error();
void launch_engram_gather(DevMat tables, Caches c, int S, int T, int p0, int slots, float* e, cudaStream_t st);
void launch_engram_vhist(const float* kv, Caches c, int site, int nsites, int S, int T, int p0, cudaStream_t st);
void launch_engram_conv(const float* taps, Caches c, int site, int nsites, int S, int T, int p0, float* v, cudaStream_t st);
// u [M][768]; gates [M][24]: the gate projections the post block's gates
// come from (see launch_mhc_gates).
// The same CTA then applies the engram gate (ekv [M][1536] and evals
// [M][768] of the layer's site, or both NULL), the input norm, and A8 of the
// normed row: x1 [M][768] (the residual), act/sx for the q|k|v|gate matmul.
void launch_mhc_read(LayerW w, int lane, const float* xs, int M, float* u, float* gates, const float* ekv,
                     const float* evals, float* x1, int8_t* act, float* sx, cudaStream_t st);
// gates [M][24] holds the post block's gate projections in [4..23] after
// launch_mhc_read; this turns them into hpost [0..3] and the Sinkhorn
// matrix hres [4..19].
void launch_mhc_gates(LayerW w, int lane, int M, float* gates, cudaStream_t st);
void launch_conv_rope_kv(LayerW w, int l, const float* proj, Caches c, int S, int T, int p0, int hist_base, const float* cosr,
                         const float* sinr, float* qbuf, cudaStream_t st);
// The q|k|v|gate projection (W: one run of all 1568 rows) and the conv in
// one launch for a one-token step of 1 .. QKVG_CONV_MAX_ROWS rows, as launch_cq_gemm(W, act,
// sx, M, 1, proj, 1568, 0) then launch_conv_rope_kv(w, l, proj, c, M, 1, ..)
// compute them; cudaErrorInvalidValue (nothing launched) outside that.
constexpr int QKVG_CONV_MAX_ROWS = 4;
cudaError_t launch_qkvg_conv(DevMat W, const int8_t* act, const float* sx, int M, float* proj, LayerW w, int l, Caches c,
                             int hist_base, const float* cosr, const float* sinr, float* qbuf, cudaStream_t st);
// window: the layer's band (0 = all); sink, ring: the attention span
// (ring 0 = none; infer.rs:1749-1825).
void launch_attention(const float* qbuf, const float* proj, Caches c, int l, int S, int T, int p0, int window, int sink,
                      int ring, float* att, int8_t* act, float* sx, cudaStream_t st);
void launch_post_block(LayerW w, const float* o, const float* x1, const float* u, const float* gates, const int32_t* perm1,
                       const int32_t* perm2, int M, float* xs, cudaStream_t st);
// The post block of a layer (w) and the mHC read of the next (wn, lane
// lane_next, its engram rows ekv/evals or NULL) for the same M rows, as
// launch_post_block then launch_mhc_read compute them, in one launch:
// batches of at most one row an SM (cudaErrorInvalidValue, nothing
// launched, otherwise). u/un, x1/x1n and gates/pn may be the same buffers.
cudaError_t launch_post_mhc(LayerW w, const float* o, const float* x1, const float* u, const float* gates, const int32_t* perm1,
                            const int32_t* perm2, int M, float* xs, LayerW wn, int lane_next, float* un, float* pn, const float* ekv,
                            const float* evals, float* x1n, int8_t* act, float* sx, cudaStream_t st);
void launch_final_hidden(const float* xs, const float* final_norm, int S, int T, int all_rows, float* h, cudaStream_t st);
void launch_rope_rows(const float* table_cos, const float* table_sin, const float* sd, const float* cd, const int32_t* p0p, int T,
                      int recur, float* state, float* cosr, float* sinr, cudaStream_t st);
void launch_advance_len(int32_t* len, int T, cudaStream_t st);
void launch_hold(unsigned long long ns, cudaStream_t st);
void launch_masked_argmax(const float* logits, int S, int V, const uint8_t* allow, int32_t* next, cudaStream_t st);
// infer.rs:1195-1211: the lane mean of rows m = (s, i) of xs [M][4][768] at
// depth `depth` into cells [S][ncap][l1][768], position p0 + i.
void launch_record_cells(const float* xs, int S, int T, int p0, int depth, int l1, int ncap, float* cells, cudaStream_t st);
// heads.rs:12-61, 77-90: the head over the cells of T positions of each of
// S sequences. r [S][l1 * k][768] and pooled [S][q * 768] are scratch.
// kind 0: the embedding (project, then unit norm) into out [S][h.out];
// kind 1: the pool alone at unit norm, out [S][q * 768] (the embedding
// without an embedding head); kind 2: the projection's first value (the
// confidence logit), out [S].
void launch_probe_head(HeadW h, const float* cells, int S, int T, int ncap, int l1, int kind, float* r, float* pooled,
                       float* out, cudaStream_t st);
// The call sampler's start, per row of logits [S][V]: with the
// entries whose `allow` bit is clear read as -1e30, the max m[s] and
// z[s] = sum exp(l - m) as agent.rs:1241-1252 forms them; with those of
// `allow_order` cleared too, live[s] = how many exceed -1e30 and ids[s][0..k)
// the first k of them by (logit descending, id ascending) (agent.rs:335-343),
// -1 past live. k <= 128, V <= 65536; ex [S][V] is scratch.
// cudaErrorInvalidValue (nothing launched) otherwise.
cudaError_t launch_candidates(const float* logits, int S, int V, const uint8_t* allow, const uint8_t* allow_order, int k,
                              int32_t* ids, float* m, double* z, int32_t* live, float* ex, cudaStream_t st);

}  // namespace nd
