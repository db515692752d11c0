// The `.cact` archive on the host: reader, CQ packer, synthetic writer.
// See cact.h; reference citations are paths in the needle-rs repository.

#include "cact.h"

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstring>
#include <stdexcept>
#include <thread>

namespace nd {

static uint32_t rd32(const uint8_t* p) { uint32_t v; std::memcpy(&v, p, 4); return v; }
static uint64_t rd64(const uint8_t* p) { uint64_t v; std::memcpy(&v, p, 8); return v; }
static float bitsf(uint32_t u) { float f; std::memcpy(&f, &u, 4); return f; }
static uint32_t fbits(float f) { uint32_t u; std::memcpy(&u, &f, 4); return u; }

static const uint32_t TAG = 0x05E12A84u;     // cact.rs:18
static const uint32_t TAG_V2 = 0x05E12A83u;  // cact.rs:19
static const size_t HEADER_BYTES = 49 * 4;   // cact.rs:21
static const size_t REC_SIZE = 44;           // cact.rs:22

void cact_parse(const uint8_t* data, size_t len, CactArchive& a) {
    if (!data || len < HEADER_BYTES) throw std::runtime_error("not a complete .cact archive");
    uint32_t tag = rd32(data);
    if (tag != TAG) {
        if (tag == TAG_V2) throw std::runtime_error("this is a Needle 2 archive; Needle 3 (tag 0x05e12a84) is required");
        char buf[64];
        snprintf(buf, sizeof buf, "unknown .cact format tag 0x%08x", tag);
        throw std::runtime_error(buf);
    }
    for (int i = 0; i < 49; i++) a.h[i] = rd32(data + 4 * i);
    if (a.h[26] > 4 || a.h[31] > 16) throw std::runtime_error("corrupt .cact header");
    a.data = data;
    a.len = len;
    size_t off = HEADER_BYTES, cbn = a.h[2];
    if (cbn > len || off + cbn * 4 > len) throw std::runtime_error("truncated codebook");
    a.codebook.resize(cbn);
    for (size_t i = 0; i < cbn; i++) a.codebook[i] = bitsf(rd32(data + off + 4 * i));
    off += cbn * 4;
    a.recs.clear();
    for (uint32_t i = 0; i < a.h[1]; i++) {
        if (off + REC_SIZE > len) throw std::runtime_error("truncated directory");
        const uint8_t* b = data + off;
        CactRecord r;
        int nd = b[1];
        if (nd > 4) throw std::runtime_error("corrupt .cact record");
        r.dtype = b[0];
        if (r.dtype < 1 || r.dtype > 4) throw std::runtime_error("unknown .cact tensor dtype " + std::to_string(r.dtype));
        for (int k = 0; k < nd; k++) r.shape.push_back(rd32(b + 4 + 4 * k));
        r.offset = rd64(b + 20);
        r.nbytes = rd64(b + 28);
        r.group = rd32(b + 36);
        r.bits = rd32(b + 40);
        if (r.offset > len || r.nbytes > len - r.offset) throw std::runtime_error("tensor past the end of the archive");
        a.recs.push_back(r);
        off += REC_SIZE;
    }
}

uint16_t f32_to_f16(float f) {
    uint32_t x = fbits(f);
    uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
    uint32_t ax = x & 0x7fffffffu;
    if (ax >= 0x7f800000u) return sign | (ax > 0x7f800000u ? 0x7e00 : 0x7c00);
    if (ax >= 0x477ff000u) return sign | 0x7c00;
    if (ax < 0x38800000u) return sign | (uint16_t)std::nearbyint(bitsf(ax) * 16777216.0f);
    uint32_t h = (((ax >> 23) - 112) << 10) | ((ax & 0x7fffff) >> 13);
    uint32_t rem = ax & 0x1fff;
    if (rem > 0x1000 || (rem == 0x1000 && (h & 1))) h++;
    return sign | (uint16_t)h;
}

float f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1f, m = h & 0x3ff;
    if (e == 0) return bitsf(fbits((float)m * 5.9604644775390625e-8f) | sign);
    if (e == 31) return bitsf(sign | 0x7f800000u | (m << 13));
    return bitsf(sign | ((e + 112) << 23) | (m << 13));
}

// crates/needle-core/src/quant.rs:19-47: the Lloyd-Max Gaussian centroids as
// the reference stores them (exact f64 bit patterns; the codebook format is
// shared with every archive, so the table must be the same).
static const uint64_t LM2[4] = {0xbff81b52e4028034ull, 0xbfdce467275b97c2ull, 0x3fdcfd177c54d348ull, 0x3ff828af1c856640ull};
static const uint64_t LM3[8] = {0xc00121468f3c6b81ull, 0xbff556e7125deacaull, 0xbfe7f2e0f9d592abull, 0xbfce6e4509e1aa2cull,
                                0x3fd000bb25e4dfa5ull, 0x3fe82dc469b936a5ull, 0x3ff568607ac227c5ull, 0x40012e5beccc8fdaull};
static const uint64_t LM4[16] = {0xc005ae0f408928fbull, 0xc0005b0b8a516d54ull, 0xbff9841ff0758fc8ull, 0xbff3bbbebadac679ull,
                                 0xbfed82c6dd21f59eull, 0xbfe47717151708b5ull, 0xbfd7d9b9e4b565faull, 0xbfbd4ca474b8559bull,
                                 0x3fc2683e9154fce2ull, 0x3fd9daf49368793aull, 0x3fe586b43e57d29dull, 0x3feec3d50cbc3b33ull,
                                 0x3ff4688db93b85f1ull, 0x3ffa3164906b428full, 0x4000ace7bbde2442ull, 0x4005ed98d06f2a4aull};

std::vector<float> cq_codebook(int bits, int group) {
    double s = std::sqrt((double)group);
    if (bits == CQ_TERNARY) {  // quant.rs:14, 59: {-c, 0, c}
        const double c = 1.2240064;
        return {(float)(-c / s), (float)(0.0 / s), (float)(c / s)};
    }
    const uint64_t* t = bits == 2 ? LM2 : bits == 3 ? LM3 : bits == 4 ? LM4 : nullptr;
    if (!t) throw std::runtime_error("no CQ codebook for " + std::to_string(bits) + " bits");
    int n = 1 << bits;
    std::vector<float> out(n);
    for (int i = 0; i < n; i++) {
        double c;
        std::memcpy(&c, &t[i], 8);
        out[i] = (float)(c / s);
    }
    return out;
}

int cq_width(int bits) {
    if (bits == CQ_TERNARY) return 2;
    if (bits >= 2 && bits <= 4) return bits;
    throw std::runtime_error("CQ records of " + std::to_string(bits) + " bits are not supported");
}

int cq_centroid(int bits, int code) {
    if (bits != CQ_TERNARY) return code;
    return code == 3 ? 0 : code + 1;  // qlinear.rs:225-227
}

// quant.rs:91-115: unnormalised FWHT, then the 1/sqrt(n) scale.
static void rotate128(float* x) {
    for (int h = 1; h < 128; h *= 2)
        for (int i = 0; i < 128; i += 2 * h)
            for (int j = i; j < i + h; j++) {
                float a = x[j], b = x[j + h];
                x[j] = a + b;
                x[j + h] = a - b;
            }
    const float s = (float)(1.0 / std::sqrt(128.0));
    for (int i = 0; i < 128; i++) x[i] *= s;
}

void cq_pack(const float* w, int rows, int d, int bits, uint8_t* packed, uint16_t* norms) {
    const std::vector<float> cb = cq_codebook(bits, 128);
    const int ncb = (int)cb.size(), width = cq_width(bits), bpg = 16 * width;
    const int groups = (d + 127) / 128;
    float g[128];
    uint8_t idx[128];
    for (int r = 0; r < rows; r++) {
        for (int gi = 0; gi < groups; gi++) {
            int start = gi * 128, take = std::min(128, d - start);
            for (int i = 0; i < 128; i++) g[i] = i < take ? w[(size_t)r * d + start + i] : 0.f;
            rotate128(g);  // quant.rs:127-135
            float ss = 0.f;
            for (int i = 0; i < 128; i++) ss = ss + g[i] * g[i];
            float norm = std::sqrt(ss);
            float denom = std::fmax(norm, 1e-12f);
            for (int i = 0; i < 128; i++) {
                float x = g[i] / denom;
                int pos = 0;  // quant.rs:119-124: nearest, ties to the lower centroid
                while (pos < ncb && cb[pos] < x) pos++;
                pos = std::min(std::max(pos, 1), ncb - 1);
                int k = std::fabs(x - cb[pos - 1]) <= std::fabs(x - cb[pos]) ? pos - 1 : pos;
                // a ternary record stores centroid k as code (k + 3) % 4
                // (the inverse of qlinear.rs:225-227)
                idx[i] = (uint8_t)(bits == CQ_TERNARY ? (k + 3) % 4 : k);
            }
            norms[(size_t)r * groups + gi] = f32_to_f16(norm);
            // quant.rs:185-198: LSB-first, 8 codes per `width` bytes
            uint8_t* dst = packed + ((size_t)r * groups + gi) * bpg;
            for (int c8 = 0; c8 < 16; c8++) {
                uint32_t word = 0;
                for (int i = 0; i < 8; i++) word |= (uint32_t)idx[8 * c8 + i] << (i * width);
                for (int b = 0; b < width; b++) dst[c8 * width + b] = (uint8_t)(word >> (8 * b));
            }
        }
    }
}

void cq_codes(const uint8_t* group_codes, int width, uint8_t out[128]) {
    for (int c8 = 0; c8 < 16; c8++) {
        uint32_t word = 0;
        for (int b = 0; b < width; b++) word |= (uint32_t)group_codes[c8 * width + b] << (8 * b);
        for (int i = 0; i < 8; i++) out[8 * c8 + i] = (uint8_t)((word >> (i * width)) & ((1u << width) - 1));
    }
}

void cq_row(const uint8_t* codes, const uint16_t* norms, int groups, int in_dim, int bits, size_t r, float* out) {
    const std::vector<float> cb = cq_codebook(bits, 128);
    const int width = cq_width(bits), bpg = 16 * width;
    float fv[16];
    for (int c = 0; c < 16; c++) {
        int k = cq_centroid(bits, c);
        fv[c] = c < (1 << width) && k < (int)cb.size() ? cb[k] : 0.f;
    }
    std::vector<float> buf((size_t)groups * 128);
    uint8_t idx[128];
    for (int g = 0; g < groups; g++) {
        float norm = f16_to_f32(norms[r * groups + g]);
        cq_codes(codes + (r * groups + g) * bpg, width, idx);
        float* dst = buf.data() + g * 128;
        for (int p = 0; p < 128; p++) dst[p] = fv[idx[p]] * norm;
        rotate128(dst);
    }
    std::memcpy(out, buf.data(), sizeof(float) * in_dim);
}

float quant_i8(const float* x, int n, int8_t* q) {
    float m = 0.f;
    for (int i = 0; i < n; i++) m = std::fmax(m, std::fabs(x[i]));
    float s = m > 0.f ? m * bitsf(0x3c010204u) : 1.0f;
    float inv = 1.0f / s;
    for (int i = 0; i < n; i++) q[i] = (int8_t)std::min(std::max(std::round(x[i] * inv), -128.f), 127.f);
    return s;
}

// --------------------------------------------------------------- writer

namespace {

// SplitMix64 sub-stream per record, Box-Muller normals in double.
struct Normal {
    uint64_t s;
    bool has = false;
    double spare = 0;
    explicit Normal(uint64_t seed) : s(seed) {}
    uint64_t next() {
        s += 0x9E3779B97F4A7C15ull;
        uint64_t z = s;
        z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
        z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
        return z ^ (z >> 31);
    }
    double uniform() { return ((double)(next() >> 11) + 0.5) * (1.0 / 9007199254740992.0); }
    double normal() {
        if (has) { has = false; return spare; }
        double u1 = uniform(), u2 = uniform();
        double r = std::sqrt(-2.0 * std::log(u1)), th = 6.283185307179586 * u2;
        spare = r * std::sin(th);
        has = true;
        return r * std::cos(th);
    }
};

struct Out {
    int dtype;
    std::vector<uint32_t> shape;
    std::vector<uint8_t> blob;
    uint32_t group = 0, bits = 0;
    // generation recipe
    enum Kind { RANDOM_F16, RANDOM_CQ, PERM, VALUES } kind;
    int rows = 0, cols = 0;
    std::vector<float> perm;
};

// rng.rs:4-74, 77-88: numpy RandomState(seed).permutation.
std::vector<float> mt_perm(uint32_t seed, int n) {
    uint32_t mt[624];
    mt[0] = seed;
    for (int i = 1; i < 624; i++) mt[i] = 1812433253u * (mt[i - 1] ^ (mt[i - 1] >> 30)) + (uint32_t)i;
    int idx = 624;
    auto next = [&]() {
        if (idx >= 624) {
            for (int i = 0; i < 624; i++) {
                uint32_t y = (mt[i] & 0x80000000u) | (mt[(i + 1) % 624] & 0x7fffffffu);
                uint32_t v = mt[(i + 397) % 624] ^ (y >> 1);
                if (y & 1) v ^= 0x9908b0dfu;
                mt[i] = v;
            }
            idx = 0;
        }
        uint32_t y = mt[idx++];
        y ^= y >> 11;
        y ^= (y << 7) & 0x9d2c5680u;
        y ^= (y << 15) & 0xefc60000u;
        return y ^ (y >> 18);
    };
    std::vector<int> a(n);
    for (int i = 0; i < n; i++) a[i] = i;
    for (int i = n - 1; i >= 1; i--) {
        uint32_t max = (uint32_t)i, mask = max;
        mask |= mask >> 1; mask |= mask >> 2; mask |= mask >> 4; mask |= mask >> 8; mask |= mask >> 16;
        uint32_t v;
        do { v = next() & mask; } while (v > max);
        std::swap(a[i], a[v]);
    }
    return std::vector<float>(a.begin(), a.end());
}

}  // namespace

std::vector<uint8_t> synth_cact(const SynthSpec& sp) {
    const int d = 768, nh = 12, nkv = 2, qk = 48, vd = 64, lanes = 4, hn = 1024, taps = 3, rank = 8;
    const int L = sp.num_layers, nsites = (int)sp.engram_sites.size();
    const int orders[2] = {2, 3}, heads = d / (2 * 128), sub = 128, ntables = 2 * heads;
    if (L < 1 || L > 64) throw std::runtime_error("synthetic depth must be in [1, 64]");
    if (nsites > 16) throw std::runtime_error("cact header holds 16 engram sites");
    for (int s : sp.engram_sites)
        if (s < 0 || s >= L) throw std::runtime_error("engram site outside the stack");
    std::vector<Out> ts;
    size_t ncq = 0;
    auto f16 = [&](std::vector<uint32_t> shape) {
        Out o;
        o.dtype = CACT_F16;
        o.kind = Out::RANDOM_F16;
        o.shape = shape;
        o.rows = 1;
        o.cols = 1;
        for (auto v : shape) o.cols *= (int)v;
        ts.push_back(o);
    };
    auto cq = [&](int rows, int cols) {
        Out o;
        o.dtype = CACT_CQ;
        o.kind = Out::RANDOM_CQ;
        o.shape = {(uint32_t)rows, (uint32_t)cols};
        o.rows = rows;
        o.cols = cols;
        o.group = 128;
        o.bits = (uint32_t)(ncq < sp.cq_bits.size() ? sp.cq_bits[ncq] : 4);
        cq_width((int)o.bits);
        ncq++;
        ts.push_back(o);
    };
    // cact.rs:279-352, the canonical order.
    cq(sp.vocab, d);
    for (int l = 0; l < L; l++) {
        f16({(uint32_t)d});                       // ZCRMSNorm_0/scale
        cq(nh * qk, d);                           // q_proj
        cq(nkv * qk, d);                          // k_proj
        cq(nkv * vd, d);                          // v_proj
        f16({(uint32_t)taps, (uint32_t)(nh * qk)});   // q_taps
        f16({(uint32_t)taps, (uint32_t)(nkv * qk)});  // k_taps
        f16({(uint32_t)taps, (uint32_t)(nkv * vd)});  // v_taps
        f16({(uint32_t)qk});                      // q_norm
        f16({(uint32_t)qk});                      // k_norm
        cq(nh * vd, d);                           // gate_proj
        cq(d, nh * vd);                           // out_proj
        f16({(uint32_t)d});                       // post_attn_norm
        f16({1});                                 // attn_gate
        f16({(uint32_t)d});                       // pre_hada_norm
        for (int k = 0; k < 5; k++) f16({(uint32_t)hn});  // d1 d2 b2 d3 d4
        for (int k = 0; k < 6; k++) f16({32, 32});        // w1a w1b w2a w2b w3a w3b
        f16({(uint32_t)d, (uint32_t)rank});       // cond_v
        f16({(uint32_t)rank, (uint32_t)hn});      // cond_u
    }
    f16({(uint32_t)L}); f16({(uint32_t)L}); f16({(uint32_t)L});  // mhc_a_pre/post/res
    f16({(uint32_t)L, (uint32_t)lanes});                        // mhc_b_pre
    f16({(uint32_t)L, (uint32_t)lanes});                        // mhc_b_post
    f16({(uint32_t)L, (uint32_t)(lanes * lanes)});              // mhc_b_res
    cq(L * lanes, lanes * d);                                   // mhc_phi_pre
    cq(L * lanes, lanes * d);                                   // mhc_phi_post
    cq(L * lanes * lanes, lanes * d);                           // mhc_phi_res
    for (uint32_t seed : {11u, 13u}) {
        Out o;
        o.dtype = CACT_F32;
        o.kind = Out::PERM;
        o.shape = {(uint32_t)hn};
        o.perm = mt_perm(seed, hn);
        ts.push_back(o);
    }
    for (int s = 0; s < nsites; s++) {
        cq(ntables * sp.engram_slots, sub);  // engrams_s/embedding
        cq(d, d);                            // key_proj
        cq(d, d);                            // value_proj
        f16({4, (uint32_t)d});               // taps
    }
    f16({(uint32_t)d});  // final_norm
    // cact.rs:362-392: the probe heads present, in HEAD_KEYS order (codes 1
    // embedding, 2 confidence, 3 router), after a manifest of their codes.
    std::vector<int> head_codes;
    for (int code = 1; code <= 3; code++)
        if ((sp.heads_mask >> code) & 1) head_codes.push_back(code);
    if (!head_codes.empty()) {
        const int l1 = L + 1, k = sp.probes, q = sp.queries;
        auto values = [&](std::vector<float> v) {
            Out o;
            o.dtype = CACT_F16;
            o.kind = Out::VALUES;
            o.shape = {(uint32_t)v.size()};
            o.perm = v;
            ts.push_back(o);
        };
        values(std::vector<float>(head_codes.begin(), head_codes.end()));
        for (int code : head_codes) {
            const int out = code == 1 ? sp.embedding_dim : code == 2 ? 1 : 3;
            cq(l1 * k, d);                                           // probes [(L+1) * k, d]
            f16({(uint32_t)l1, (uint32_t)k});                        // gain
            cq(q, d);                                                // query
            f16({(uint32_t)q, (uint32_t)l1, (uint32_t)k});           // row_bias
            cq(out, q * d);                                          // proj [out, q * d]
            f16({(uint32_t)out});                                    // bias
            if (code == 3) values({0.90f, 0.00f, 0.60f});            // calibration
        }
    }

    // Fill the blobs, records in parallel, each from its own sub-stream.
    std::atomic<size_t> next(0);
    auto work = [&]() {
        for (;;) {
            size_t i = next.fetch_add(1);
            if (i >= ts.size()) return;
            Out& o = ts[i];
            Normal rng(sp.seed * 0x100000001B3ull + 0x51ED270B2A6F1C3Dull * (i + 1));
            if (o.kind == Out::VALUES) {
                o.blob.resize(o.perm.size() * 2);
                for (size_t k2 = 0; k2 < o.perm.size(); k2++) {
                    uint16_t h = f32_to_f16(o.perm[k2]);
                    std::memcpy(&o.blob[2 * k2], &h, 2);
                }
            } else if (o.kind == Out::PERM) {
                o.blob.resize(o.perm.size() * 4);
                std::memcpy(o.blob.data(), o.perm.data(), o.blob.size());
            } else if (o.kind == Out::RANDOM_F16) {
                o.blob.resize((size_t)o.cols * 2);
                for (int k = 0; k < o.cols; k++) {
                    uint16_t h = f32_to_f16((float)(sp.std * rng.normal()));
                    std::memcpy(&o.blob[2 * k], &h, 2);
                }
            } else {
                std::vector<float> w((size_t)o.rows * o.cols);
                for (auto& v : w) v = (float)(sp.std * rng.normal());
                int groups = (o.cols + 127) / 128;
                size_t npk = (size_t)o.rows * groups * 16 * cq_width((int)o.bits);
                o.blob.resize(npk + (size_t)o.rows * groups * 2);
                std::vector<uint16_t> norms((size_t)o.rows * groups);
                cq_pack(w.data(), o.rows, o.cols, (int)o.bits, o.blob.data(), norms.data());
                std::memcpy(o.blob.data() + npk, norms.data(), norms.size() * 2);
            }
        }
    };
    unsigned nth = std::max(1u, std::min(16u, std::thread::hardware_concurrency()));
    std::vector<std::thread> th;
    for (unsigned k = 0; k < nth; k++) th.emplace_back(work);
    for (auto& t : th) t.join();

    // cact.rs:399-475
    std::vector<float> cbs;
    for (int b : {2, 3, 4}) {
        auto c = cq_codebook(b, 128);
        cbs.insert(cbs.end(), c.begin(), c.end());
    }
    // config.rs:448-482 for this geometry.
    auto kv_window = [&]() -> uint32_t {
        const int per_layer = nkv * qk + nkv * vd + (nkv * qk / 32 + nkv * vd / 32) * 4;
        const int per_site = d + (d / 32) * 4;
        const long budget = 11L * 1024 * 1024 + 512 * 1024;
        int n_global = 0;
        for (int l = 0; l < L; l++) n_global += (sp.global_mask >> l) & 1;
        if (sp.sliding_window > 0) {
            long local = std::min(sp.sliding_window, sp.max_seq_len);
            long fixed = ((long)(L - n_global) * per_layer + (long)nsites * per_site) * local;
            if (n_global == 0) return fixed <= budget ? sp.max_seq_len : (uint32_t)std::max(160L, local);
            long num = budget - fixed, den = (long)n_global * per_layer;
            auto fdiv = [](long a, long b) { long q = a / b; if ((a % b != 0) && ((a < 0) != (b < 0))) q--; return q; };
            long ctx = fdiv(fdiv(num, den), 32) * 32;
            return (uint32_t)std::max(160L, std::min(ctx, (long)sp.max_seq_len));
        }
        long per_pos = (long)L * per_layer + (long)nsites * per_site;
        long window = (budget / per_pos) / 32 * 32;
        return (uint32_t)std::max(160L, std::min(window, (long)sp.max_seq_len));
    }();
    std::vector<uint32_t> hdr = {TAG, (uint32_t)ts.size(), (uint32_t)cbs.size(), kv_window, 8, (uint32_t)sp.vocab, 0,
                                 (uint32_t)d, (uint32_t)nh, (uint32_t)nkv, (uint32_t)L, (uint32_t)qk, (uint32_t)vd,
                                 (uint32_t)sp.max_seq_len, (uint32_t)hn, (uint32_t)lanes, (uint32_t)sp.sliding_window,
                                 (uint32_t)(sp.global_mask & 0xffffffffu), (uint32_t)(sp.global_mask >> 32), (uint32_t)taps,
                                 (uint32_t)sp.engram_slots, (uint32_t)sub, (uint32_t)ntables, 4, 3, 0, 2};
    hdr.push_back(orders[0]);
    hdr.push_back(orders[1]);
    hdr.push_back(0);
    hdr.push_back(0);
    hdr.push_back((uint32_t)nsites);
    for (int k = 0; k < 16; k++) hdr.push_back(k < nsites ? (uint32_t)sp.engram_sites[k] : 0);
    hdr.push_back(fbits(100000.0f));
    if (hdr.size() != 49) throw std::runtime_error("header size");
    std::vector<uint8_t> buf(HEADER_BYTES);
    std::memcpy(buf.data(), hdr.data(), HEADER_BYTES);
    for (float v : cbs) {
        uint32_t u = fbits(v);
        buf.insert(buf.end(), (uint8_t*)&u, (uint8_t*)&u + 4);
    }
    size_t pos = buf.size() + ts.size() * REC_SIZE;
    std::vector<uint64_t> offs;
    for (auto& t : ts) {
        pos = (pos + 63) & ~(size_t)63;
        offs.push_back(pos);
        pos += t.blob.size();
    }
    for (size_t i = 0; i < ts.size(); i++) {
        uint8_t r[REC_SIZE] = {0};
        r[0] = (uint8_t)ts[i].dtype;
        r[1] = (uint8_t)ts[i].shape.size();
        for (size_t k = 0; k < ts[i].shape.size() && k < 4; k++) std::memcpy(r + 4 + 4 * k, &ts[i].shape[k], 4);
        uint64_t nb = ts[i].blob.size();
        std::memcpy(r + 20, &offs[i], 8);
        std::memcpy(r + 28, &nb, 8);
        std::memcpy(r + 36, &ts[i].group, 4);
        std::memcpy(r + 40, &ts[i].bits, 4);
        buf.insert(buf.end(), r, r + REC_SIZE);
    }
    for (size_t i = 0; i < ts.size(); i++) {
        buf.resize(offs[i], 0);
        buf.insert(buf.end(), ts[i].blob.begin(), ts[i].blob.end());
    }
    return buf;
}

}  // namespace nd
