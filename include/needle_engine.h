/*
 * needle_engine.h — the model-level C ABI under needle.h: the contract the
 * reference's engine crate gives its agent, CLI and benches (Model, Session,
 * head logits), made batched so one call advances many independent
 * sequences on one GPU. Plain pointers and sizes only.
 *
 * Each entry names the reference interface it replaces (file:line in
 * needle-rs). A batch holds S sequences that are fed in lockstep: every call
 * gives each sequence the same number of new tokens, so they share positions.
 * A batch is driven by one host thread at a time.
 *
 * Pointers: with ND_DEVICE in `flags` the id/mask/output pointers are device
 * pointers on the model's GPU and the call is asynchronous on the batch's
 * stream; otherwise they are host pointers, copied in and out inside the
 * call, which returns when the results are in host memory.
 */
#ifndef NEEDLE_ENGINE_H
#define NEEDLE_ENGINE_H

#ifdef __cplusplus
extern "C" {
#endif

typedef struct nd_model nd_model;
typedef struct nd_batch nd_batch;

enum { ND_DEVICE = 1 };

/* crates/needle-engine/src/model.rs:150-160 (`Outputs`). */
enum {
    ND_OUT_NONE = 0,        /* Outputs::None */
    ND_OUT_LAST_LOGITS = 1, /* Outputs::LastLogits: [S][out_rows] */
    ND_OUT_LAST_HIDDEN = 2, /* Outputs::LastHidden: [S][d_model] */
    ND_OUT_ALL_LOGITS = 3,  /* Outputs::AllLogits: [S][t][out_rows] */
    ND_OUT_HIDDEN = 4       /* Outputs::Hidden: [S][t][d_model] */
};

/* crates/needle-engine/src/loader.rs:40-59 with weights.rs:314-497
 * (Weights::from_archive_mode, fast) and model.rs:248-253 (Model::quantized):
 * parse the archive, upload its packed matrices and small weights to GPU
 * `device`, build the int8 gate projection and RoPE tables. The archive
 * bytes are only read during the call. 0 on success, -1 on error. */
int nd_model_load(const unsigned char* cact, unsigned long long n, int device, nd_model** out);
void nd_model_free(nd_model* m);

/* crates/needle-core/src/cact.rs:173-202 (Header::to_config): dims[0..9] =
 * vocab, out_rows, d_model, num_layers, num_heads, num_kv_heads,
 * qk_head_dim, v_head_dim, max_seq_len. */
int nd_model_dims(const nd_model* m, int* dims);

/* model.rs:264-274 (Model::session), for `num_seqs` sequences of up to
 * `max_len` positions each. `max_len` must lie in [1, max_seq_len] and be
 * at most 8192 (the attention kernel holds 32 key chunks of 256); beyond
 * that the call fails with a message, as a too-long session does. */
int nd_batch_new(nd_model* m, int num_seqs, int max_len, nd_batch** out);
void nd_batch_free(nd_batch* b);

/* model.rs:72-74 (Session::len): positions every sequence has been fed. */
int nd_batch_len(const nd_batch* b);

/* Session::attend (crates/needle-engine/src/model.rs:63-66, infer.rs:
 * 1749-1825) for every sequence of the batch: each query sees the first
 * `sink` positions within its layer's band, then the positions from
 * max(chunk end - ring, sink) on (the engine's ring, which the band does
 * not cut), as the agent sets it (agent.rs:583-588: sink = the static
 * prefix, ring = the header's kv_window). ring = 0 restores plain
 * attention. Rollbacks are not served, so every position in those runs
 * still holds its keys (the batch's cache keeps all max_len positions). */
int nd_batch_set_attend(nd_batch* b, int sink, int ring);

/* Session::rollback (model.rs:81-113, infer.rs:1055-1077): drop the last
 * n <= 32 positions of every sequence without recomputing; the next feed
 * continues from there (conv and engram histories, RoPE rows and KV of the
 * kept positions stay). Fails, changing nothing, when under the batch's
 * attention span a kept position's ring slot holds a dropped position (the
 * reference would skip that key and re-feed it, which is not served). */
int nd_batch_rollback(nd_batch* b, int n);

/* Session::rewind_zeroed (model.rs:116-126, infer.rs:1039-1053): forget
 * positions len.. as the engine's context-overflow re-feed does: the KV
 * cache keeps what it holds, the conv history and RoPE rows start over.
 * The same refusal as nd_batch_rollback. */
int nd_batch_rewind_zeroed(nd_batch* b, int len);

/* Session::truncate (model.rs:128-145): drop everything past len; up to 32
 * positions by nd_batch_rollback, more by feeding the first len tokens to
 * fresh sessions again (which, as in the reference, have no attention
 * span). */
int nd_batch_truncate(nd_batch* b, int len);

/* model.rs:304-306 (Model::forward) through infer.rs:1105-1131
 * (forward_native): feed ids[S][t] to every sequence in the engine's chunks
 * of at most 32, writing `outputs` to out (may be NULL for ND_OUT_NONE).
 * Returns the rows written per sequence, -1 on error. */
int nd_batch_forward(nd_batch* b, const int* ids, int t, int outputs, float* out, int flags);

/* The greedy decode loop of crates/needle-cli/src/main.rs:577-581 and
 * generate.rs:110-125, with the agent's ban (agent.rs:1114-1127): for each
 * sequence take the first index of the maximum of its last logits after the
 * ids its mask disallows read -1e30 (allow_bits [S][ceil(out_rows/8)], bit
 * set = allowed, LSB first; NULL allows all), write it to next_ids[S], and
 * feed it as one decode step. Needs a preceding forward with logits. */
int nd_batch_step(nd_batch* b, const unsigned char* allow_bits, int* next_ids, int flags);

/* infer.rs:1016 (NatState::last_hidden): each sequence's final normed hidden
 * state of the last position a forward returned outputs for, [S][d_model]. */
int nd_batch_last_hidden(nd_batch* b, float* out, int flags);

/* infer.rs:1135-1141 (Model::head_logits): logits of h[rows][d_model] with
 * the decode kernel, out[rows][out_rows]. */
int nd_head_logits(nd_batch* b, const float* h, int rows, float* out, int flags);

/* infer.rs:1145-1166 (Model::head_logits_sparse): one row h[d_model]; the
 * ids are scored with the single-row kernel, every other entry is NEG
 * (0xf149f2ca). out[out_rows]. Host pointers. */
int nd_head_logits_sparse(nd_batch* b, const float* h, const int* ids, int n, float* out);

/* The start of the agent's grammar-constrained call step, per sequence,
 * over logits[S][out_rows] (NULL = the batch's last logits; the agent's
 * sparse-logit rows, agent.rs:390-420, come in this way)
 * (crates/needle-engine/src/agent.rs:295-343):
 * entries whose bit in `allow` is clear read -1e30 (the step's bans; NULL =
 * none), and over that m[s] = the max and z[s] = sum exp(l - m) as
 * softmax_stats forms them (agent.rs:1241-1252: four f32 lanes of the
 * engine's exp over whole groups of four, then the remainder in f64).
 * Entries whose bit in `allow_order` is also clear (the call step's further
 * bans; NULL = none) leave the candidates: live[s] = how many logits
 * exceed -1e30 and ids[s][0..k) the first k of them by logit, lowest id
 * first on ties (the top-128 partial selection and sort, agent.rs:335-343),
 * -1 past live. 1 <= k <= 128; masks [S][ceil(out_rows/8)], bit set =
 * allowed. The grammar's accept test that walks these candidates stays on
 * the host. Host pointers, or device pointers with ND_DEVICE. */
int nd_batch_candidates(nd_batch* b, const float* logits, const unsigned char* allow, const unsigned char* allow_order,
                        int k, int* ids, float* m, double* z, int* live, int flags);

/* needle_embed's computation after tokenizing (crates/needle-engine/src/
 * heads.rs:63-90, agent.rs:259-263) for every sequence of a fresh batch
 * (nothing fed yet): ids[S][T] are fed in chunks of 32 recording the lane
 * mean of the residual stream at every position and depth (the cells,
 * infer.rs:1195-1211), then the probe pool of the embedding head,
 * projected and scaled to unit norm (without an embedding head, the
 * confidence head's pool at unit norm). out[S][dim]; with out == NULL only
 * *dim is set. Fails without a probe head ("this archive carries no probe
 * head"). The batch keeps the T fed positions. Host or device pointers
 * (ND_DEVICE). */
int nd_batch_embed(nd_batch* b, const int* ids, int T, float* out, int* dim, int flags);

/* heads.rs:68-74 (confidence_logit) the same way: out[S] = the confidence
 * head's logit for each sequence of a fresh batch. */
int nd_batch_confidence(nd_batch* b, const int* ids, int T, float* out, int flags);

/* The CUDA stream a batch's work runs on (a cudaStream_t); no counterpart
 * in the reference, which runs on the CPU. */
void* nd_batch_stream(nd_batch* b);

/* crates/needle-core/src/quant.rs:233-256 (cq_pack, group 128) at bits 2,
 * 3, 4 or 5 (ternary; quant.rs:11-12): w[rows][d] to codes[rows][G * 16 *
 * width] (G = ceil(d/128), width = bits, 2 for ternary; LSB-first) and f16
 * norms[rows][G]. The reference's packer takes bits 4 only; the other widths
 * are written in the layout its loader reads (qlinear.rs:220-236). */
int nd_cq_pack(const float* w, int rows, int d, int bits, unsigned char* codes, unsigned short* norms);

/* Test and benchmark support: one CQ matrix (codes [out][6][16 * width],
 * f16 norms [out][6] as nd_cq_pack writes them at `bits`; in_dim 768) on GPU
 * `device`, and the engine's matmul of host rows x[M][768] into y[M][out]:
 * each row quantized as QAct::new (qlinear.rs:152-207), then the decode
 * combine (qlinear.rs:340-350) when T == 1, else the prefill combine
 * (qlinear.rs:353-363) over consecutive sequences of T rows (M a multiple
 * of T). With reps > 0 and ms != NULL it also times reps back-to-back runs
 * (A8 + matmul, inputs resident) and stores the mean in *ms. */
typedef struct nd_cqmat nd_cqmat;
int nd_cqmat_new(int device, const unsigned char* codes, const unsigned short* norms, int out, int in_dim, int bits,
                 nd_cqmat** out_mat);
void nd_cqmat_free(nd_cqmat* mat);
int nd_cqmat_apply(nd_cqmat* mat, const float* x, int M, int T, float* y, int reps, float* ms);
/* Benchmark support: the matmul alone (no A8), launched back to back over
 * the n matrices in turn, `reps` rounds after one untimed round, on the
 * activations the last nd_cqmat_apply of mats[0] quantized (M <= its rows).
 * When the matrices together exceed L2 every launch streams its weights
 * from HBM. *ms = mean time per launch. The matrices share device and
 * shape. */
int nd_cqmat_time_rotating(nd_cqmat* const* mats, int n, int M, int T, int reps, float* ms);

/* crates/needle-core/src/cact.rs:399-475 (pack) over random-init Needle 3
 * weights: every tensor ~N(0, std^2), seeded; CQ matrices, f16 small
 * weights, MT19937 Hadamard permutations. Shape knobs let tests shrink the
 * model (num_layers, vocab, engram_slots, sliding_window; engram_sites is
 * a bit mask of layers, global_mask likewise). cq_bits[i] is the record
 * bits (2, 3, 4, 5 = ternary) of the i-th CQ record in record order, 4 past
 * n_cq_bits (a mixed-width archive; the reference's packer writes one
 * width). heads_mask bit c appends probe head c (1 embedding, 2
 * confidence, 3 router; cact.rs:354-392: 4 probes a depth, 4 queries, the
 * embedding head 128 wide). With out == NULL returns the byte size in
 * *len; else writes up to cap bytes. */
int nd_synth_cact(int num_layers, int vocab, int engram_slots, int sliding_window, unsigned long long global_mask,
                  unsigned long long engram_sites, unsigned long long seed, float std, const int* cq_bits, int n_cq_bits,
                  unsigned heads_mask, unsigned char* out, unsigned long long cap, unsigned long long* len);

/* Kernel launches this process has issued (all batches, all devices); no
 * counterpart in the reference. */
long long nd_launch_count(void);

/* Launch sites whose kernels can be timed with CUDA events on the batch's
 * stream (no counterpart in the reference): nd_batch_time_site(b, site)
 * starts recording every launch of that site (clearing earlier records;
 * ND_SITE_NONE stops), nd_batch_site_time() waits for the stream and
 * returns the summed kernel time and the number of launches. Two sites share
 * launches in small batches: with at most one row an SM, each layer's post
 * block launch also runs the next layer's mHC read (ND_SITE_POST covers
 * both; ND_SITE_MHC times layer 0's alone), and one-token steps of up to
 * four sequences run the q|k|v|gate projection with the conv (ND_SITE_QKVG
 * covers both; ND_SITE_CONV records none). */
enum {
    ND_SITE_NONE = 0,
    ND_SITE_QKVG = 1,      /* q|k|v|gate projection */
    ND_SITE_OUT = 2,       /* attention out projection */
    ND_SITE_LM_HEAD = 3,   /* tied lm_head logits */
    ND_SITE_ENGRAM_KV = 4, /* engram key|value projection */
    ND_SITE_ATTENTION = 5, /* int8 KV attention + gate */
    ND_SITE_POST = 6,      /* post block: norms, Hadamard MLP, Sinkhorn, mHC write */
    ND_SITE_MHC = 7,       /* mHC read, engram gate, input norm, A8 */
    ND_SITE_CONV = 8       /* conv taps, head norm, RoPE, int8 KV write */
};
int nd_batch_time_site(nd_batch* b, int site);
int nd_batch_site_time(nd_batch* b, double* total_ms, int* launches);

/* No counterpart in the reference. nd_head_logits without any allocation,
 * for callers that cannot call cudaMalloc (their GPU memory belongs to
 * another allocator, or they must not take cudaMalloc's implicit device
 * synchronisation): logits of h[rows][d_model] into out[rows][out_rows] with
 * the decode kernel, both device pointers on the model's GPU, queued on
 * `stream` (a cudaStream_t; NULL is the legacy default stream) and not
 * waited for. The int8 activations live in one static device array of the
 * library, so rows is limited to 1..64; larger requests return -1 with the
 * reason in nd_last_error(). The first call on each device looks up that
 * array's device address, so make it before capturing any stream into a
 * CUDA graph. All calls share the array: calls whose work overlaps on the
 * GPU (other streams, other threads) race; the array keeps the last call's
 * contents, none of which the next call reads before writing. */
int nd_head_logits_noalloc(const nd_model* m, const float* h, int rows, float* out, void* stream);

/* The fused row ops of a layer as standalone kernels (BASELINE's fused-ops
 * sweep; in the forward pass they are fused into larger kernels). Device
 * pointers, queued on `stream` (a cudaStream_t; NULL = the legacy default
 * stream) and not waited for; 0 on success, -1 with nd_last_error().
 * Float pointers must be 16-byte aligned. */

/* infer.rs:426-443 (zcn, the zero-centred RMSNorm) with infer.rs:372-417
 * (dot16): out[t] = fma(x[t] r, s, x[t] r), r = 1 / sqrt(dot16(x[t],
 * x[t]) / 768 + 1e-6), for rows x[T][768] and weights s[768]. */
int nd_op_zcn(const float* x, const float* s, int T, float* out, void* stream);

/* The rotary embedding of a chunk's rows (infer.rs:1474-1483 with the
 * tables of infer.rs:938-946 and 1716-1744) at positions 0 .. T-1: x[T][672]
 * holds 12 query heads then 2 key heads of 48; in each, x[f] and x[f + 24]
 * (f < 24) rotate by the angle freq[f] * t, freq[f] = powf(theta,
 * f * (-2 / 48)). out may equal x. */
int nd_op_rope(const float* x, int T, float theta, float* out, void* stream);

/* infer.rs:2463-2496 (silu_native): out[i] = x[i] / (nexp(-x[i]) + 1) for
 * n elements (the Hadamard MLP's activation). */
int nd_op_silu(const float* x, long long n, float* out, void* stream);

/* qlinear.rs:309-323 (QMat::row) of the model's token embedding for each of
 * ids[T] (device int32): out[T][d_model], the codes dequantized by their
 * f16 group norms and rotated back (without the forward's sqrt(d_model)
 * scale). An id outside [0, vocab) gives a row of zeros. */
int nd_op_gather(const nd_model* m, const int* ids, int T, float* out, void* stream);

/* The last failure on this thread (empty if none). */
const char* nd_last_error(void);

/* Test support: copy an internal per-row buffer of the last forward
 * ("xs", "u", "p", "x1", "proj", "qbuf", "att", "o", "h", "logits", or the
 * same names snapped after layer `layer` when nd_batch_debug_layer(b, layer)
 * was set, prefixed "snap."). Returns the float count, -1 if unknown. */
int nd_batch_debug(nd_batch* b, const char* name, float* out, long long cap);
int nd_batch_debug_layer(nd_batch* b, int layer);

#ifdef __cplusplus
}
#endif

#endif /* NEEDLE_ENGINE_H */
