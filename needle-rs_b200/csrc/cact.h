// The `.cact` Needle 3 archive (format tag 0x05E12A84), host side: reader,
// CQ-4 packer and the random-init model writer the benchmarks load.
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
};

// A random-init Needle 3 archive: every tensor ~N(0, std^2) drawn in record
// order from one seeded stream, CQ-4 matrices packed by the reference's
// quantizer (crates/needle-core/src/quant.rs:233-256), small weights as f16,
// Hadamard permutations from MT19937 seeds 11 and 13 (rng.rs:77-88), written
// in cact.rs:279-352's canonical record order by cact.rs:399-475's packer.
std::vector<uint8_t> synth_cact(const SynthSpec& spec);

// quant.rs:233-256 (bits = 4, group = 128).
void cq_pack4(const float* w, int rows, int d, uint8_t* packed, uint16_t* norms);

// IEEE binary16 round-to-nearest-even, as the `half` crate 2.7.1 converts.
uint16_t f32_to_f16(float f);
float f16_to_f32(uint16_t h);

// qlinear.rs:309-323 (QMat::row): row r of a CQ-4 matrix dequantized,
// `fvals[code] * norm` per group then rotated, truncated to in_dim.
void cq_row(const uint8_t* codes, const uint16_t* norms, int groups, int in_dim, size_t r, float* out);

// qlinear.rs:77-88: absmax int8 with s = amax * K127, round half away.
float quant_i8(const float* x, int n, int8_t* q);

// quant.rs:50-68: the unit-sphere CQ codebook (bits 2, 3, 4).
std::vector<float> cq_codebook(int bits, int group);

}  // namespace nd
