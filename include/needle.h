/*
 * needle.h — the Needle 3 engine's C API, unchanged from the reference.
 *
 * Each declaration replaces the same-named entry of needle-rs's C ABI
 * (crates/needle-ffi/src/lib.rs); the line ranges are cited per function.
 * One process-global engine; calls are serialised by an internal mutex.
 * Negative returns are failures and needle_last_error() says why.
 *
 * This library runs the model on an NVIDIA B200 (sm_100a). needle_load is
 * complete. The agent layer above the model (tokenizer, chat template,
 * grammar-constrained tool calling) is not part of this engine yet:
 * needle_init, needle_complete and needle_embed report that through
 * needle_last_error and return -1.
 */
#ifndef NEEDLE_H
#define NEEDLE_H

#ifdef __cplusplus
extern "C" {
#endif

/* lib.rs:59-77. Parses a .cact archive (the bytes are read during the call
 * only) and uploads its weights to the GPU. 0 on success, -1 on error. */
int needle_load(const unsigned char* cact, unsigned long long n);

/* lib.rs:81-99. Binds a toolset; returns the static-prefix token count. */
int needle_init(const char* system_prompt, const char* tools_json, const char* tool_index_path);

/* lib.rs:116-141. One agent turn into out; the byte length, -1 on error (the
 * message also written to out), -2 when out_capacity is too small. */
int needle_complete(const char* input, int max_new_tokens, char* out, int out_capacity);

/* lib.rs:146-171. The retrieval embedding; out == NULL returns its length. */
int needle_embed(const char* input, float* out, int out_capacity);

/* lib.rs:173-178. Rewinds the conversation to the bound static prefix. */
void needle_reset(void);

/* lib.rs:180-183. The last failure's message (empty if none). */
const char* needle_last_error(void);

#ifdef __cplusplus
}
#endif

#endif /* NEEDLE_H */
