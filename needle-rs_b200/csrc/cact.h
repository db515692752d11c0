// The `.cact` Needle 3 archive (format tag 0x05E12A84), host side: reader,
// CQ packer and the random-init model writer the benchmarks load.
//
// Layout follows crates/needle-core/src/cact.rs:1-120 (196-byte header, f32
// codebooks, 44-byte records, 64-byte aligned blobs in canonical order).
#pragma once

#include <cstddef>
#include <cstdint>
#include <string>
#include <vector>

namespace nd {

enum CactDtype { CACT_F16 = 1, CACT_F32 = 2, CACT_CQ = 3, CACT_RAW = 4 };

// Record `bits` value of ternary CQ codes (quant.rs:11-12): 2-bit crumbs,
// code 3 the first centroid and codes 0, 1 the others (qlinear.rs:225-227).
constexpr int CQ_TERNARY = 5;

struct CactRecord {
    int dtype = 0;
    std::vector<uint32_t> shape;
    uint64_t offset = 0, nbytes = 0;
    uint32_t group = 0, bits = 0;
};

struct CactArchive {
    const uint8_t* data = nullptr;
    size_t len = 0;
    uint32_t h[49] = {0};
    std::vector<float> codebook;
    std::vector<CactRecord> recs;
    const uint8_t* bytes(size_t i) const { return data + recs[i].offset; }
};

// crates/needle-core/src/cact.rs:122-165, 230-243, 580-601. Throws
// std::runtime_error with the reference's messages on corrupt input.
void cact_parse(const uint8_t* data, size_t len, CactArchive& out);

// Geometry of a synthetic archive. Defaults are Needle 3's
// (crates/needle-core/src/config.rs:60-103); tests shrink the depth, vocab and
// engram slots to keep the CPU oracle fast.
struct SynthSpec {
    int num_layers = 20;
    int vocab = 16384;
    int engram_slots = 18432;
    int sliding_window = 1024;
    int max_seq_len = 4096;
    uint64_t global_mask = (1ull << 4) | (1ull << 9) | (1ull << 14) | (1ull << 19);
    std::vector<int> engram_sites = {3, 7, 11, 15, 19};
    uint64_t seed = 0;
    float std = 0.02f;
    // Code width of each CQ record in record order (2, 3, 4 or CQ_TERNARY);
    // records past the end of the list are 4-bit.
    std::vector<int> cq_bits;
    // Probe heads to append (bit `code`: 1 embedding, 2 confidence, 3
    // router), with k probes per depth, q queries, and the embedding head's
    // width (config.rs:27-33, 72-77).
    unsigned heads_mask = 0;
    int probes = 4, queries = 4, embedding_dim = 128;
};

// A random-init Needle 3 archive: every tensor ~N(0, std^2) drawn in record
// order from one seeded stream, CQ matrices packed by the reference's
// quantizer (crates/needle-core/src/quant.rs:233-256), small weights as f16,
// Hadamard permutations from MT19937 seeds 11 and 13 (rng.rs:77-88), written
// in cact.rs:279-352's canonical record order by cact.rs:399-475's packer.
std::vector<uint8_t> synth_cact(const SynthSpec& spec);

// quant.rs:233-256 (group 128) at `bits` = 2, 3, 4 or CQ_TERNARY: nearest
// centroid of the width's codebook, codes packed LSB-first, 8 per `width`
// bytes (16 * width bytes a group). The reference's packer stops at 4 bits;
// the other widths follow the layout its loader reads (quant.rs:259-287,
// qlinear.rs:220-236).
void cq_pack(const float* w, int rows, int d, int bits, uint8_t* packed, uint16_t* norms);

// Bits a code takes in memory for a record's `bits` (ternary packs at 2);
// throws for widths the engine does not read.
int cq_width(int bits);
// The codebook entry a code selects (ternary remaps, qlinear.rs:225-227).
int cq_centroid(int bits, int code);
// quant.rs:208-225: the 128 codes of one group, `width` bits each.
void cq_codes(const uint8_t* group_codes, int width, uint8_t out[128]);

// IEEE binary16 round-to-nearest-even, as the `half` crate 2.7.1 converts.
uint16_t f32_to_f16(float f);
float f16_to_f32(uint16_t h);

// qlinear.rs:309-323 (QMat::row): row r of a CQ matrix of record width
// `bits` dequantized, `fvals[code] * norm` per group then rotated,
// truncated to in_dim.
void cq_row(const uint8_t* codes, const uint16_t* norms, int groups, int in_dim, int bits, size_t r, float* out);

// qlinear.rs:77-88: absmax int8 with s = amax * K127, round half away.
float quant_i8(const float* x, int n, int8_t* q);

// quant.rs:50-68: the unit-sphere CQ codebook (bits 2, 3, 4, CQ_TERNARY).
std::vector<float> cq_codebook(int bits, int group);

}  // namespace nd
