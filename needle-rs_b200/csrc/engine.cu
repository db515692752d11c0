// The Needle 3 engine on one GPU: archive upload, batched sequence state and
// the forward sequencing of the reference's native path, behind the C ABI of
// include/needle_engine.h and include/needle.h.

#include <cmath>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <stdexcept>
#include <string>
#include <vector>

#include "cact.h"
#include "kernels.h"
#include "needle.h"
#include "needle_engine.h"

namespace nd {

static thread_local std::string g_err;

#define CK(x)                                                                                                          \
    do {                                                                                                               \
        cudaError_t e_ = (x);                                                                                          \
        if (e_ != cudaSuccess) throw std::runtime_error(std::string("CUDA error: ") + cudaGetErrorString(e_) + " (" #x ")"); \
    } while (0)

struct Config {
    int vocab, out_vocab, d, nh, nkv, L, qk, vd, max_seq, hada_n, lanes, sw;
    uint64_t global_mask;
    int taps, eslots, esub, ntables, etaps, edil, eseed;
    std::vector<int> orders, sites;
    float theta;
    int out_rows() const { return out_vocab > 0 ? out_vocab : vocab; }
    int window(int l) const { return (sw > 0 && !((global_mask >> l) & 1)) ? sw : 0; }
};

// A projection as the engine runs it: consecutive runs of output rows, one
// DevMat (one codebook) each; a uniform archive has one run per projection.
struct Linear {
    std::vector<DevMat> runs;
    int out = 0;
};

struct Model {
    int device = 0;
    Config c;
    std::vector<void*> allocs;
    DevMat embedding;
    DevMat head;  // the embedding's first out_rows() rows: the tied lm_head
    std::vector<LayerW> layers;
    std::vector<Linear> qkvg, out;  // per layer
    std::vector<DevMat> etables;
    std::vector<Linear> ekv;
    HeadW heads[3];  // weights.rs:60-76: embedding, confidence, router
    bool has_head[3] = {false, false, false};
    std::vector<const float*> etaps;
    std::vector<int> site_of_layer;
    const int32_t *perm1 = nullptr, *perm2 = nullptr;
    const float* final_norm = nullptr;
    const float *rope_cos = nullptr, *rope_sin = nullptr, *sd = nullptr, *cd = nullptr;
    std::vector<float> h_sd, h_cd;

    template <class T>
    T* upload(const T* h, size_t n) {
        void* p = nullptr;
        CK(cudaMalloc(&p, n * sizeof(T) + 16));
        allocs.push_back(p);
        CK(cudaMemcpy(p, h, n * sizeof(T), cudaMemcpyHostToDevice));
        return (T*)p;
    }
    ~Model() {
        cudaSetDevice(device);
        for (void* p : allocs) cudaFree(p);
    }
};

// cact.rs:173-202
static Config config_of(const CactArchive& a) {
    Config c;
    const uint32_t* h = a.h;
    c.vocab = h[5]; c.out_vocab = h[6]; c.d = h[7]; c.nh = h[8]; c.nkv = h[9]; c.L = h[10];
    c.qk = h[11]; c.vd = h[12]; c.max_seq = h[13]; c.hada_n = h[14]; c.lanes = h[15]; c.sw = h[16];
    c.global_mask = (uint64_t)h[17] | ((uint64_t)h[18] << 32);
    c.taps = h[19]; c.eslots = h[20]; c.esub = h[21]; c.ntables = h[22]; c.etaps = h[23]; c.edil = h[24]; c.eseed = h[25];
    for (uint32_t i = 0; i < h[26]; i++) c.orders.push_back(h[27 + i]);
    for (uint32_t i = 0; i < h[31]; i++) c.sites.push_back(h[32 + i]);
    std::memcpy(&c.theta, &h[48], 4);
    return c;
}

struct Cursor {
    const CactArchive& a;
    size_t i = 0;
    const CactRecord& next(int dtype) {
        if (i >= a.recs.size()) throw std::runtime_error("archive ends before the model does");
        const CactRecord& r = a.recs[i++];
        if (r.dtype != dtype) throw std::runtime_error("archive tensor " + std::to_string(i - 1) + " has the wrong dtype");
        return r;
    }
};

static std::vector<float> small_f32(const CactArchive& a, Cursor& cur, size_t expect) {
    size_t idx = cur.i;
    const CactRecord& r = cur.a.recs.at(idx);
    std::vector<float> v;
    if (r.dtype == CACT_F16) {
        cur.i++;
        v.resize(r.nbytes / 2);
        for (size_t k = 0; k < v.size(); k++) {
            uint16_t h;
            std::memcpy(&h, a.bytes(idx) + 2 * k, 2);
            v[k] = f16_to_f32(h);
        }
    } else if (r.dtype == CACT_F32) {
        cur.i++;
        v.resize(r.nbytes / 4);
        std::memcpy(v.data(), a.bytes(idx), r.nbytes);
    } else {
        throw std::runtime_error("archive tensor " + std::to_string(idx) + " is not a small f16/f32 weight");
    }
    if (expect && v.size() < expect) throw std::runtime_error("archive tensor " + std::to_string(idx) + " is too small");
    return v;
}

struct HostMat {
    std::vector<uint8_t> codes;   // [out][groups][16 * width]
    std::vector<uint16_t> norms;  // [out][groups] f16
    int out = 0, in_dim = 0, groups = 0;
    int bits = 4;  // the record's bits: 2, 3, 4 or CQ_TERNARY
};

// qlinear.rs:220-236 (group 128; code widths 2, 3, 4 and ternary)
static HostMat host_mat(const CactArchive& a, Cursor& cur, int in_dim) {
    const CactRecord& r = cur.next(CACT_CQ);
    if (r.group != 128) throw std::runtime_error("CQ group size " + std::to_string(r.group) + " is not supported");
    if (r.shape.size() != 2 || (int)r.shape[1] != in_dim) throw std::runtime_error("CQ matrix has the wrong input width");
    HostMat m;
    m.bits = (int)r.bits;
    const int width = cq_width(m.bits);
    m.out = (int)r.shape[0];
    m.in_dim = in_dim;
    m.groups = (in_dim + 127) / 128;
    size_t nc = (size_t)m.out * m.groups * 16 * width, nn = (size_t)m.out * m.groups;
    if (r.nbytes < nc + nn * 2) throw std::runtime_error("CQ record is truncated");
    const uint8_t* b = a.bytes(cur.i - 1);
    m.codes.assign(b, b + nc);
    m.norms.resize(nn);
    std::memcpy(m.norms.data(), b + nc, nn * 2);
    return m;
}

// qlinear.rs:211-216, 244-265: a record width's codebook as the kernels
// read it: code -> int8 value (ternary codes remapped, codes past the
// codebook 0), its scale, and code -> f32 value.
static void code_table(int bits, DevMat& d) {
    const std::vector<float> cb = cq_codebook(bits, 128);
    float mx = 0.f;
    for (float v : cb) mx = std::fmax(mx, std::fabs(v));
    uint32_t k127u = 0x3c010204u;
    float k127;
    std::memcpy(&k127, &k127u, 4);
    const float cbs = mx > 0.f ? mx * k127 : 1.0f;
    const float inv = 1.0f / cbs;
    int8_t vals[16] = {0};
    d.width = cq_width(bits);
    for (int c = 0; c < 16; c++) {
        const int k = cq_centroid(bits, c);
        const bool in = c < (1 << d.width) && k < (int)cb.size();
        vals[c] = in ? (int8_t)std::min(std::max(std::round(cb[k] * inv), -128.f), 127.f) : 0;
        d.fvals[c] = in ? cb[k] : 0.f;
    }
    std::memcpy(d.vals4, vals, 16);
    d.cbs = cbs;
}

// A matrix on the device: the archive's codes and norms, its codebook, and
// (for the projections that run as matmuls) the codes expanded through the
// int8 codebook into lane-major groups (see DevMat::w8).
static DevMat to_dev(Model& m, const HostMat& h, bool expand) {
    DevMat d;
    d.codes = m.upload(h.codes.data(), h.codes.size());
    d.norms = m.upload(h.norms.data(), h.norms.size());
    d.out = h.out;
    d.in_dim = h.in_dim;
    d.groups = h.groups;
    code_table(h.bits, d);
    if (expand) {
        int8_t vals[16];
        std::memcpy(vals, d.vals4, 16);
        int slot[128];
        for (int p = 0; p < 128; p++) slot[p] = lane_major_slot(p);
        const int K = h.groups * 128, bpg = 16 * d.width;
        std::vector<int8_t> w((size_t)h.out * K);
        uint8_t idx[128];
        for (size_t r = 0; r < (size_t)h.out; r++)
            for (int g = 0; g < h.groups; g++) {
                cq_codes(h.codes.data() + (r * h.groups + g) * bpg, d.width, idx);
                int8_t* dst = w.data() + r * K + g * 128;
                for (int p = 0; p < 128; p++) dst[slot[p]] = vals[idx[p]];
            }
        d.w8 = m.upload(w.data(), w.size());
    }
    return d;
}

// QLinear::new (qlinear.rs:500-518): parts side by side over one input;
// neighbours of the same record bits share a codebook and become one run,
// and every part must share the code width (the activation layout).
static Linear to_linear(Model& m, const std::vector<const HostMat*>& parts) {
    Linear lin;
    for (size_t i = 0; i < parts.size();) {
        if (cq_width(parts[i]->bits) != cq_width(parts[0]->bits))
            throw std::runtime_error("fused parts must share a code width");
        size_t j = i;
        HostMat run;
        while (j < parts.size() && parts[j]->bits == parts[i]->bits) {
            const HostMat& p = *parts[j++];
            if (run.out == 0) {
                run = p;
            } else {
                run.out += p.out;
                run.codes.insert(run.codes.end(), p.codes.begin(), p.codes.end());
                run.norms.insert(run.norms.end(), p.norms.begin(), p.norms.end());
            }
        }
        lin.runs.push_back(to_dev(m, run, true));
        lin.out += run.out;
        i = j;
    }
    return lin;
}

// Every run of a projection into y[m][col0 ..] (ldy wide), one launch each.
static void linear(const Linear& lin, const int8_t* act, const float* sx, int M, int T, float* y, int ldy,
                   cudaStream_t st) {
    int col = 0;
    for (const DevMat& d : lin.runs) {
        CK(launch_cq_gemm(d, act, sx, M, T, y, ldy, col, st));
        col += d.out;
    }
}

// weights.rs:314-497 (record walk, fast mode), infer.rs:938-962 (Tables).
static Model* load_model(const uint8_t* bytes, size_t n, int device) {
    CactArchive a;
    cact_parse(bytes, n, a);
    std::unique_ptr<Model> mp(new Model());
    Model& m = *mp;
    m.device = device;
    CK(cudaSetDevice(device));
    Config& c = m.c;
    c = config_of(a);
    if (c.lanes != 4 || c.hada_n != 1024 || c.taps != 3 || c.qk != 48 || c.vd != 64 || c.d != 768 || c.nh != 12 ||
        c.nkv != 2 || c.etaps != 4 || c.edil != 3 || c.esub != 128 || c.ntables != 6 || c.orders.size() != 2 ||
        c.orders[0] != 2 || c.orders[1] != 3 || c.eseed != 0)
        throw std::runtime_error("the native path covers the shipped Needle 3 geometry only");
    if (c.L < 1 || c.L > 64 || c.vocab < 1 || c.out_rows() > c.vocab || c.max_seq < 1)
        throw std::runtime_error("corrupt .cact header");
    Cursor cur{a};
    const int d = c.d;
    HostMat emb = host_mat(a, cur, d);
    if (emb.out != c.vocab) throw std::runtime_error("embedding shape does not match the header");
    m.embedding = to_dev(m, emb, true);
    m.head = m.embedding;
    m.head.out = c.out_rows();
    m.layers.resize(c.L);
    m.qkvg.resize(c.L);
    m.out.resize(c.L);
    for (int l = 0; l < c.L; l++) {
        LayerW& w = m.layers[l];
        std::memset(&w, 0, sizeof w);
        w.norm_in = m.upload(small_f32(a, cur, d).data(), d);
        HostMat q = host_mat(a, cur, d), k = host_mat(a, cur, d), v = host_mat(a, cur, d);
        auto qt = small_f32(a, cur, 3 * 576), kt = small_f32(a, cur, 3 * 96), vt = small_f32(a, cur, 3 * 128);
        w.q_taps = m.upload(qt.data(), qt.size());
        w.k_taps = m.upload(kt.data(), kt.size());
        w.v_taps = m.upload(vt.data(), vt.size());
        w.q_norm = m.upload(small_f32(a, cur, 48).data(), 48);
        w.k_norm = m.upload(small_f32(a, cur, 48).data(), 48);
        HostMat g = host_mat(a, cur, d), o = host_mat(a, cur, 768);
        if (q.out != 576 || k.out != 96 || v.out != 128 || g.out != 768 || o.out != d)
            throw std::runtime_error("attention projection shapes do not match the header");
        m.qkvg[l] = to_linear(m, {&q, &k, &v, &g});
        m.out[l] = to_linear(m, {&o});
        w.post_norm = m.upload(small_f32(a, cur, d).data(), d);
        w.attn_gate = small_f32(a, cur, 1)[0];
        w.pre_hada = m.upload(small_f32(a, cur, d).data(), d);
        auto d1 = small_f32(a, cur, d), d2 = small_f32(a, cur, 1024), b2 = small_f32(a, cur, 1024),
             d3 = small_f32(a, cur, 1024), d4 = small_f32(a, cur, d);
        w.d1 = m.upload(d1.data(), d1.size());
        w.d2 = m.upload(d2.data(), d2.size());
        w.b2 = m.upload(b2.data(), b2.size());
        w.d3 = m.upload(d3.data(), d3.size());
        w.d4 = m.upload(d4.data(), d4.size());
        for (int k6 = 0; k6 < 6; k6++) w.kron[k6] = m.upload(small_f32(a, cur, 1024).data(), 1024);
        {
            // cond_v [768][8] as the post block's conditioning chains read
            // it: chain (set, k) = row 8 set + k holds cond_v[set + 4 n][k]
            // at column n (n < 192), rows COND_LD floats apart
            const auto cv = small_f32(a, cur, (size_t)d * 8);
            std::vector<float> cx((size_t)32 * COND_LD, 0.f);
            for (int set = 0; set < 4; set++)
                for (int k = 0; k < 8; k++)
                    for (int n = 0; n < 192; n++) cx[(size_t)(set * 8 + k) * COND_LD + n] = cv[(size_t)(set + 4 * n) * 8 + k];
            w.cond_v = m.upload(cx.data(), cx.size());
        }
        w.cond_u = m.upload(small_f32(a, cur, 8 * 1024).data(), 8 * 1024);
    }
    const int nl = c.lanes, nc = nl * d;
    auto a_pre = small_f32(a, cur, c.L), a_post = small_f32(a, cur, c.L), a_res = small_f32(a, cur, c.L);
    auto b_pre = small_f32(a, cur, c.L * nl), b_post = small_f32(a, cur, c.L * nl), b_res = small_f32(a, cur, c.L * nl * nl);
    HostMat phi[3] = {host_mat(a, cur, nc), host_mat(a, cur, nc), host_mat(a, cur, nc)};
    if (phi[0].out != c.L * nl || phi[1].out != c.L * nl || phi[2].out != c.L * nl * nl)
        throw std::runtime_error("mHC projection shapes do not match the header");
    std::vector<float> row(nc);
    for (int l = 0; l < c.L; l++) {
        LayerW& w = m.layers[l];
        w.a_pre = a_pre[l]; w.a_post = a_post[l]; w.a_res = a_res[l];
        for (int j = 0; j < 4; j++) { w.b_pre[j] = b_pre[l * 4 + j]; w.b_post[j] = b_post[l * 4 + j]; }
        for (int j = 0; j < 16; j++) w.b_res[j] = b_res[l * 16 + j];
        // weights.rs:380-391 + 493 (pre | post | res rows dequantized),
        // infer.rs:852-866 (each row requantized to int8 with its scale)
        std::vector<int8_t> q(24 * (size_t)nc);
        std::vector<float> s(24);
        int k = 0;
        const int base[3] = {l * 4, l * 4, l * 16}, cnt[3] = {4, 4, 16};
        for (int part = 0; part < 3; part++)
            for (int rr = 0; rr < cnt[part]; rr++, k++) {
                cq_row(phi[part].codes.data(), phi[part].norms.data(), phi[part].groups, nc, phi[part].bits, base[part] + rr,
                       row.data());
                s[k] = quant_i8(row.data(), nc, q.data() + (size_t)k * nc);
            }
        w.phi_q = m.upload(q.data(), q.size());
        w.phi_s = m.upload(s.data(), s.size());
    }
    auto p1 = small_f32(a, cur, 1024), p2 = small_f32(a, cur, 1024);
    if ((int)p1.size() != c.hada_n || (int)p2.size() != c.hada_n) throw std::runtime_error("Hadamard permutations do not match hada_n");
    std::vector<int32_t> ip1(1024), ip2(1024);
    for (int j = 0; j < 1024; j++) {
        ip1[j] = (int32_t)p1[j];
        ip2[j] = (int32_t)p2[j];
        if (ip1[j] < 0 || ip1[j] >= 1024 || ip2[j] < 0 || ip2[j] >= 1024) throw std::runtime_error("corrupt Hadamard permutation");
    }
    m.perm1 = m.upload(ip1.data(), 1024);
    m.perm2 = m.upload(ip2.data(), 1024);
    for (size_t s = 0; s < c.sites.size(); s++) {
        HostMat t = host_mat(a, cur, 128);
        if (t.out != c.ntables * c.eslots) throw std::runtime_error("engram table shape does not match the header");
        HostMat k = host_mat(a, cur, d), v = host_mat(a, cur, d);
        m.etables.push_back(to_dev(m, t, false));
        m.ekv.push_back(to_linear(m, {&k, &v}));
        auto taps = small_f32(a, cur, 4 * (size_t)d);
        m.etaps.push_back(m.upload(taps.data(), taps.size()));
    }
    m.final_norm = m.upload(small_f32(a, cur, d).data(), d);
    // weights.rs:422-469: probe heads between final_norm and the tokenizer
    size_t tok_index = a.recs.size();
    for (size_t r = 0; r < a.recs.size(); r++)
        if (a.recs[r].dtype == CACT_RAW) { tok_index = r; break; }
    if (cur.i < tok_index) {
        const int l1 = c.L + 1;
        // any tensor as f32 (cact.rs:620-630): CQ matrices dequantized by row
        auto dense = [&](int in_dim, int* rows) -> std::vector<float> {
            const CactRecord& r = a.recs.at(cur.i);
            if (r.dtype != CACT_CQ) {
                std::vector<float> v = small_f32(a, cur, 0);
                if (rows) *rows = r.shape.empty() ? 1 : (int)r.shape[0];
                return v;
            }
            HostMat hm = host_mat(a, cur, in_dim);
            std::vector<float> v((size_t)hm.out * in_dim);
            for (int row = 0; row < hm.out; row++)
                cq_row(hm.codes.data(), hm.norms.data(), hm.groups, in_dim, hm.bits, row, v.data() + (size_t)row * in_dim);
            if (rows) *rows = hm.out;
            return v;
        };
        std::vector<float> manifest = small_f32(a, cur, 1);
        for (float code : manifest) {
            const int ci = (int)std::lround(code);
            if (ci < 1 || ci > 3) throw std::runtime_error("unknown probe head code " + std::to_string(ci));
            HeadW h;
            int prow = 0, qrow = 0, orow = 0;
            std::vector<float> probes = dense(d, &prow), gain = dense(0, nullptr), query = dense(d, &qrow);
            std::vector<float> row_bias = dense(0, nullptr);
            h.q = qrow;
            h.k = (int)(gain.size() / l1);
            std::vector<float> proj = dense(h.q * d, &orow), bias = dense(0, nullptr);
            h.out = orow;
            if (ci == 3) small_f32(a, cur, 3);  // the router's calibration
            if (h.k < 1 || probes.size() != (size_t)l1 * h.k * d || gain.size() != (size_t)l1 * h.k ||
                query.size() != (size_t)h.q * d || row_bias.size() != (size_t)h.q * l1 * h.k ||
                proj.size() != (size_t)h.out * h.q * d || bias.size() != (size_t)h.out)
                throw std::runtime_error("probe head rows do not match the depth");
            h.probes = m.upload(probes.data(), probes.size());
            h.gain = m.upload(gain.data(), gain.size());
            h.query = m.upload(query.data(), query.size());
            h.row_bias = m.upload(row_bias.data(), row_bias.size());
            h.proj = m.upload(proj.data(), proj.size());
            h.bias = m.upload(bias.data(), bias.size());
            m.heads[ci - 1] = h;
            m.has_head[ci - 1] = true;
        }
    }
    m.site_of_layer.assign(c.L, -1);
    for (size_t s = 0; s < c.sites.size(); s++) {
        if (c.sites[s] < 0 || c.sites[s] >= c.L) throw std::runtime_error("engram site outside the stack");
        m.site_of_layer[c.sites[s]] = (int)s;
    }
    // infer.rs:938-946 with the reference's non-Apple libm stand-ins
    // (infer.rs:83-102): f32 results of f64 pow / sincos, rounded once.
    const int half = c.qk / 2;
    float coef = -2.0f / (float)c.qk;
    std::vector<float> freq(half);
    m.h_sd.resize(half);
    m.h_cd.resize(half);
    for (int f = 0; f < half; f++) {
        freq[f] = (float)std::pow((double)c.theta, (double)((float)f * coef));
        double sv, cv;
        sincos((double)freq[f], &sv, &cv);
        m.h_sd[f] = (float)sv;
        m.h_cd[f] = (float)cv;
    }
    std::vector<float> tc((size_t)c.max_seq * half), ts((size_t)c.max_seq * half);
    for (int p = 0; p < c.max_seq; p++)
        for (int f = 0; f < half; f++) {
            double sv, cv;
            sincos((double)(freq[f] * (float)p), &sv, &cv);
            tc[(size_t)p * half + f] = (float)cv;
            ts[(size_t)p * half + f] = (float)sv;
        }
    m.rope_cos = m.upload(tc.data(), tc.size());
    m.rope_sin = m.upload(ts.data(), ts.size());
    m.sd = m.upload(m.h_sd.data(), half);
    m.cd = m.upload(m.h_cd.data(), half);
    set_constants((float)(1.0 / std::sqrt(128.0)));
    CK(cudaGetLastError());
    CK(cudaDeviceSynchronize());
    return mp.release();
}

// ----------------------------------------------------------------- batch

// A captured decode step: argmax under the mask, then the one-token forward.
struct StepGraph {
    cudaGraphExec_t exec = nullptr;
    long long kernels = 0;  // kernels one replay launches
    int hist_base = 0;      // the conv-history start baked into the capture
};

struct Batch {
    Model* m = nullptr;
    int S = 0, cap = 0, Mmax = 0;
    cudaStream_t st = nullptr;
    // The engram sites depend only on the tokens, so each chunk runs them on
    // a second stream, forked after the tokens are written; layer l's mHC
    // read waits for its site's event.
    cudaStream_t st2 = nullptr;
    cudaEvent_t ev_fork = nullptr;
    std::vector<cudaEvent_t> ev_site;
    // The post block's gates (hpost, Sinkhorn) depend only on the mHC read,
    // so each layer computes them on a third stream while its matmuls and
    // attention run; the post block waits for them.
    cudaStream_t st3 = nullptr;
    std::vector<cudaEvent_t> ev_mhc, ev_gates;
    int len = 0;          // positions fed to every sequence
    int hist_base = 0;    // first position whose pre-tap row the conv may read
    bool rope_valid = false;
    // the attention span (sink, ring) of every sequence (model.rs:63-66);
    // ring 0: none
    int attend_sink = 0, attend_ring = 0;
    // the reference's slot map (infer.rs:1015-1023, 1768-1776): the
    // position each KV slot last received, kept on the host to tell when a
    // rollback would leave a kept position's slot to a dropped one
    std::vector<int64_t> slot_pos;
    int rope_from = 0;  // first position whose RoPE row the ring still holds
    bool have_logits = false;
    int logits_rows = 0;
    int debug_layer = -1;
    Caches c{};
    std::vector<void*> allocs;
    float *xs, *u, *p, *x1, *proj, *qbuf, *att, *o, *e, *ekv, *evals, *cosr, *sinr, *rope_state, *h, *logits = nullptr;
    int8_t *act, *act_e;  // A8 rows of the layer chain / of the engram stream
    float *sx, *sx_e;
    int32_t *ids, *next;
    int32_t* d_len;  // device copy of len (Caches::len)
    uint8_t* masks;
    // the call sampler's buffers (nd_batch_candidates), made on first use
    // the probe heads' inputs and scratch (nd_batch_embed), made on use
    float *cells = nullptr, *head_r = nullptr, *head_pool = nullptr, *head_out = nullptr;
    int cells_cap = 0;       // positions per sequence the cells buffer holds
    bool recording = false;  // chunk() records cells while set
    float *clogits = nullptr, *cex = nullptr;
    uint8_t *cmask1 = nullptr, *cmask2 = nullptr;
    int32_t *cids = nullptr, *clive = nullptr;
    float* cm = nullptr;
    double* cz = nullptr;
    size_t logits_cap = 0;
    std::map<std::string, std::pair<float*, size_t>> snaps;
    int last_rows = 0, last_T = 0;
    int time_site = 0;                 // launch site timed with events (ND_SITE_*)
    bool graphs = true;                // replay decode steps as CUDA graphs (NEEDLE_GRAPHS=0 turns off)
    StepGraph graph[2];                // without / with a mask
    std::vector<cudaEvent_t> evs;
    size_t ev_used = 0;

    template <class T>
    T* alloc(size_t n) {
        void* p = nullptr;
        CK(cudaMalloc(&p, n * sizeof(T) + 64));
        allocs.push_back(p);
        CK(cudaMemsetAsync(p, 0, n * sizeof(T) + 64, st));
        return (T*)p;
    }
    ~Batch() {
        cudaSetDevice(m->device);
        if (st) cudaStreamSynchronize(st);
        for (void* p : allocs) cudaFree(p);
        if (logits) cudaFree(logits);
        for (auto& kv : snaps) cudaFree(kv.second.first);
        for (auto e : evs) cudaEventDestroy(e);
        for (auto& g : graph)
            if (g.exec) cudaGraphExecDestroy(g.exec);
        if (st2) cudaStreamSynchronize(st2);
        if (st3) cudaStreamSynchronize(st3);
        for (auto e : ev_site) cudaEventDestroy(e);
        for (auto e : ev_mhc) cudaEventDestroy(e);
        for (auto e : ev_gates) cudaEventDestroy(e);
        if (st3) cudaStreamDestroy(st3);
        if (ev_fork) cudaEventDestroy(ev_fork);
        if (st2) cudaStreamDestroy(st2);
        if (st) cudaStreamDestroy(st);
    }
};

static Batch* batch_new(Model* m, int S, int max_len) {
    const Config& c = m->c;
    if (S < 1) throw std::runtime_error("a batch needs at least one sequence");
    if (max_len < 1 || max_len > c.max_seq) throw std::runtime_error("max_len must be in [1, max_seq_len]");
    if (max_len > ATT_MAX_KEYS) throw std::runtime_error("max_len above 8192 positions: the attention kernel holds 32 key chunks");
    CK(cudaSetDevice(m->device));
    std::unique_ptr<Batch> bp(new Batch());
    Batch& b = *bp;
    b.m = m;
    b.S = S;
    b.cap = max_len;
    b.Mmax = S * 32;
    CK(cudaStreamCreateWithFlags(&b.st, cudaStreamNonBlocking));
    CK(cudaStreamCreateWithFlags(&b.st2, cudaStreamNonBlocking));
    CK(cudaEventCreateWithFlags(&b.ev_fork, cudaEventDisableTiming));
    if (const char* g = getenv("NEEDLE_GRAPHS")) b.graphs = atoi(g) != 0;
    const int L = c.L, nsites = (int)c.sites.size();
    b.ev_site.resize(nsites);
    for (auto& e : b.ev_site) CK(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    CK(cudaStreamCreateWithFlags(&b.st3, cudaStreamNonBlocking));
    b.ev_mhc.resize(L);
    b.ev_gates.resize(L);
    for (auto& e : b.ev_mhc) CK(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    for (auto& e : b.ev_gates) CK(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    const size_t M = b.Mmax;
    b.c.S = S;
    b.c.L = L;
    b.c.cap = max_len;
    b.c.k8 = b.alloc<int8_t>((size_t)S * L * 2 * max_len * 48);
    b.c.ks = b.alloc<float>((size_t)S * L * 2 * max_len);
    b.c.vgroups = (max_len + 3) / 4;
    b.c.v8 = b.alloc<int8_t>((size_t)S * L * 2 * b.c.vgroups * 256);
    b.c.vs = b.alloc<float>((size_t)S * L * 2 * max_len);
    b.c.hist = b.alloc<float>((size_t)S * L * HIST_RING * 800);
    b.c.ev8 = b.alloc<int8_t>((size_t)S * std::max(nsites, 1) * ENG_RING * 768);
    b.c.evs = b.alloc<float>((size_t)S * std::max(nsites, 1) * ENG_RING * 24);
    b.c.tokens = b.alloc<int32_t>((size_t)S * max_len);
    b.d_len = b.alloc<int32_t>(1);
    b.c.len = b.d_len;
    b.xs = b.alloc<float>(M * 3072);
    b.u = b.alloc<float>(M * 768);
    b.p = b.alloc<float>(M * 24);
    b.x1 = b.alloc<float>(M * 768);
    b.proj = b.alloc<float>(M * 1568);
    b.qbuf = b.alloc<float>(M * 576);
    b.att = b.alloc<float>(M * 768);
    b.o = b.alloc<float>(M * 768);
    b.e = b.alloc<float>(M * 768);
    b.ekv = b.alloc<float>((size_t)std::max(nsites, 1) * M * 1536);
    b.evals = b.alloc<float>((size_t)std::max(nsites, 1) * M * 768);
    b.cosr = b.alloc<float>(32 * 24);
    b.sinr = b.alloc<float>(32 * 24);
    b.rope_state = b.alloc<float>((size_t)ROPE_RING * 48);
    b.h = b.alloc<float>(M * 768);
    b.act = b.alloc<int8_t>(M * 768);
    b.sx = b.alloc<float>(M * 8);
    b.act_e = b.alloc<int8_t>(M * 768);
    b.sx_e = b.alloc<float>(M * 8);
    b.ids = b.alloc<int32_t>(M);
    b.next = b.alloc<int32_t>(S);
    b.masks = b.alloc<uint8_t>((size_t)S * ((c.out_rows() + 7) / 8));
    CK(cudaStreamSynchronize(b.st));
    return bp.release();
}

static void ensure_logits(Batch& b, size_t rows) {
    size_t need = rows * (size_t)b.m->c.out_rows();
    if (need <= b.logits_cap) return;
    if (b.logits) CK(cudaFree(b.logits));
    b.logits = nullptr;
    CK(cudaMalloc(&b.logits, need * sizeof(float)));
    b.logits_cap = need;
}

// An event on the launching stream around each launch of the timed site.
static void tick(Batch& b, int site, cudaStream_t on = nullptr) {
    if (b.time_site != site) return;
    if (b.ev_used == b.evs.size()) {
        cudaEvent_t e;
        CK(cudaEventCreate(&e));
        b.evs.push_back(e);
    }
    CK(cudaEventRecord(b.evs[b.ev_used++], on ? on : b.st));
}

static void snap(Batch& b, const char* name, const float* src, size_t n) {
    auto it = b.snaps.find(name);
    if (it == b.snaps.end() || it->second.second < n) {
        if (it != b.snaps.end()) cudaFree(it->second.first);
        float* p = nullptr;
        CK(cudaMalloc(&p, n * sizeof(float)));
        b.snaps[name] = {p, n};
    }
    b.snaps[name].second = n;
    CK(cudaMemcpyAsync(b.snaps[name].first, src, n * sizeof(float), cudaMemcpyDeviceToDevice, b.st));
}

// infer.rs:1749-1754: the KV slot of position p under the batch's span.
static int64_t slot_of(const Batch& b, int64_t p) {
    if (b.attend_ring > 0 && p >= b.attend_sink) return (p - b.attend_sink) % b.attend_ring + b.attend_sink;
    return p;
}

// infer.rs:1768-1776: positions p0 .. p0 + T now hold their slots.
static void mark_slots(Batch& b, int64_t p0, int T) {
    for (int64_t p = p0; p < p0 + T; p++) {
        const int64_t sl = slot_of(b, p);
        if ((int64_t)b.slot_pos.size() <= sl) b.slot_pos.resize(sl + 1, -1);
        b.slot_pos[sl] = p;
    }
}

// Whether dropping positions len.. would leave a kept position (< len)
// whose slot a dropped one holds: the reference then skips that key and
// re-feeds from it (infer.rs:1078-1100), which this engine does not serve.
static bool stale_below(const Batch& b, int64_t len) {
    for (size_t sl = 0; sl < b.slot_pos.size(); sl++)
        if (b.slot_pos[sl] >= len && (int64_t)sl < len) return true;
    return false;
}

// infer.rs:1168-1240 (chunk_native) for every sequence's chunk of T tokens
// at positions len .. len + T - 1; ids are device int32 [S][T].
static int chunk(Batch& b, const int32_t* ids, int T, int outputs) {
    Model& m = *b.m;
    const Config& c = m.c;
    const int S = b.S, M = S * T, p0 = b.len, nsites = (int)c.sites.size();
    cudaStream_t st = b.st;
    if (p0 + T > b.cap) throw std::runtime_error("sequence exceeds the batch's max_len");
    launch_write_tokens(ids, S, T, p0, b.c, st);
    mark_slots(b, p0, T);
    // infer.rs:1720: the recurrence serves one token right after the newest
    launch_rope_rows(m.rope_cos, m.rope_sin, m.sd, m.cd, b.d_len, T, (T == 1 && b.rope_valid) ? 1 : 0, b.rope_state, b.cosr,
                     b.sinr, st);
    // infer.rs:1244-1328, on the engram stream
    if (nsites > 0) {
        cudaStream_t s2 = b.st2;
        CK(cudaEventRecord(b.ev_fork, st));
        CK(cudaStreamWaitEvent(s2, b.ev_fork, 0));
        for (int s = 0; s < nsites; s++) {
            float* kv = b.ekv + (size_t)s * b.Mmax * 1536;
            launch_engram_gather(m.etables[s], b.c, S, T, p0, c.eslots, b.e, s2);
            launch_prep_act(b.e, 768, 768, M, b.act_e, b.sx_e, s2);
            tick(b, ND_SITE_ENGRAM_KV, s2);
            linear(m.ekv[s], b.act_e, b.sx_e, M, T, kv, 1536, s2);
            tick(b, ND_SITE_ENGRAM_KV, s2);
            launch_engram_vhist(kv, b.c, s, nsites, S, T, p0, s2);
            launch_engram_conv(m.etaps[s], b.c, s, nsites, S, T, p0, b.evals + (size_t)s * b.Mmax * 768, s2);
            CK(cudaEventRecord(b.ev_site[s], s2));
        }
    }
    launch_embed(m.embedding, ids, M, b.xs, st);
    if (b.recording) launch_record_cells(b.xs, S, T, p0, 0, c.L + 1, b.cells_cap, b.cells, st);
    // batches of at most one row an SM run each layer's post block and the
    // next layer's mHC read in one launch (the cells a recording batch
    // keeps, and the debug snapshots, read xs and the layer's buffers
    // before or after that launch as they would around the post block)
    const bool fuse_post_mhc = M <= device_sm_count();
    bool mhc_done = false;  // this layer's mHC read ran with the last post block
    for (int l = 0; l < c.L; l++) {
        const LayerW& w = m.layers[l];
        const int lane = l % 4, site = m.site_of_layer[l];
        if (!mhc_done) {
            if (site >= 0) CK(cudaStreamWaitEvent(st, b.ev_site[site], 0));
            tick(b, ND_SITE_MHC);
            launch_mhc_read(w, lane, b.xs, M, b.u, b.p, site >= 0 ? b.ekv + (size_t)site * b.Mmax * 1536 : nullptr,
                            site >= 0 ? b.evals + (size_t)site * b.Mmax * 768 : nullptr, b.x1, b.act, b.sx, st);
            tick(b, ND_SITE_MHC);
        }
        CK(cudaEventRecord(b.ev_mhc[l], st));
        CK(cudaStreamWaitEvent(b.st3, b.ev_mhc[l], 0));
        launch_mhc_gates(w, lane, M, b.p, b.st3);
        CK(cudaEventRecord(b.ev_gates[l], b.st3));
        if (T == 1 && M <= QKVG_CONV_MAX_ROWS && m.qkvg[l].runs.size() == 1) {
            // a one-token step of a few sequences: the projection and the
            // conv in one launch (its time counts as the q|k|v|gate site's)
            tick(b, ND_SITE_QKVG);
            CK(launch_qkvg_conv(m.qkvg[l].runs[0], b.act, b.sx, M, b.proj, w, l, b.c, b.hist_base, b.cosr, b.sinr, b.qbuf, st));
            tick(b, ND_SITE_QKVG);
        } else {
            tick(b, ND_SITE_QKVG);
            linear(m.qkvg[l], b.act, b.sx, M, T, b.proj, 1568, st);
            tick(b, ND_SITE_QKVG);
            tick(b, ND_SITE_CONV);
            launch_conv_rope_kv(w, l, b.proj, b.c, S, T, p0, b.hist_base, b.cosr, b.sinr, b.qbuf, st);
            tick(b, ND_SITE_CONV);
        }
        tick(b, ND_SITE_ATTENTION);
        launch_attention(b.qbuf, b.proj, b.c, l, S, T, p0, c.window(l), b.attend_sink, b.attend_ring, b.att, b.act, b.sx, st);
        tick(b, ND_SITE_ATTENTION);
        tick(b, ND_SITE_OUT);
        linear(m.out[l], b.act, b.sx, M, T, b.o, 768, st);
        tick(b, ND_SITE_OUT);
        CK(cudaStreamWaitEvent(st, b.ev_gates[l], 0));
        if (l == b.debug_layer) {
            snap(b, "snap.u", b.u, (size_t)M * 768);
            snap(b, "snap.p", b.p, (size_t)M * 24);
            snap(b, "snap.x1", b.x1, (size_t)M * 768);
            snap(b, "snap.proj", b.proj, (size_t)M * 1568);
            snap(b, "snap.qbuf", b.qbuf, (size_t)M * 576);
            snap(b, "snap.att", b.att, (size_t)M * 768);
            snap(b, "snap.o", b.o, (size_t)M * 768);
        }
        mhc_done = fuse_post_mhc && l + 1 < c.L;
        tick(b, ND_SITE_POST);
        if (mhc_done) {
            const int ln = l + 1, nsite = m.site_of_layer[ln];
            if (nsite >= 0) CK(cudaStreamWaitEvent(st, b.ev_site[nsite], 0));
            CK(launch_post_mhc(w, b.o, b.x1, b.u, b.p, m.perm1, m.perm2, M, b.xs, m.layers[ln], ln % 4, b.u, b.p,
                               nsite >= 0 ? b.ekv + (size_t)nsite * b.Mmax * 1536 : nullptr,
                               nsite >= 0 ? b.evals + (size_t)nsite * b.Mmax * 768 : nullptr, b.x1, b.act, b.sx, st));
        } else {
            launch_post_block(w, b.o, b.x1, b.u, b.p, m.perm1, m.perm2, M, b.xs, st);
        }
        tick(b, ND_SITE_POST);
        if (b.recording) launch_record_cells(b.xs, S, T, p0, l + 1, c.L + 1, b.cells_cap, b.cells, st);
        if (l == b.debug_layer) snap(b, "snap.xs", b.xs, (size_t)M * 3072);
    }
    // every site has joined the layer chain before the position advances
    for (int s = 0; s < nsites; s++) CK(cudaStreamWaitEvent(st, b.ev_site[s], 0));
    launch_advance_len(b.d_len, T, st);
    b.len += T;
    b.rope_valid = true;
    b.last_T = T;
    CK(cudaGetLastError());
    if (outputs == ND_OUT_NONE) return 0;
    const bool all = outputs == ND_OUT_ALL_LOGITS || outputs == ND_OUT_HIDDEN;
    const int rows = all ? M : S;
    launch_final_hidden(b.xs, m.final_norm, S, T, all ? 1 : 0, b.h, st);
    b.last_rows = rows;
    if (outputs == ND_OUT_LAST_LOGITS || outputs == ND_OUT_ALL_LOGITS) {
        ensure_logits(b, rows);
        launch_prep_act(b.h, 768, 768, rows, b.act, b.sx, st);
        // infer.rs:1135-1141: QAct of one row each, so the decode combine
        tick(b, ND_SITE_LM_HEAD);
        CK(launch_cq_gemm(m.head, b.act, b.sx, rows, 1, b.logits, c.out_rows(), 0, st));
        tick(b, ND_SITE_LM_HEAD);
        b.have_logits = true;
        b.logits_rows = rows;
    }
    CK(cudaGetLastError());
    return all ? T : 1;
}

// infer.rs:1105-1131: chunks of at most 32 from the feed start; a Last*
// request is served by the last chunk only.
static int forward(Batch& b, const int32_t* dev_ids, int t, int outputs) {
    if (t < 1) throw std::runtime_error("forward needs at least one token");
    if (outputs < 0 || outputs > 4) throw std::runtime_error("unknown outputs value");
    if ((outputs == ND_OUT_ALL_LOGITS || outputs == ND_OUT_HIDDEN) && t > 32)
        throw std::runtime_error("per-token outputs are served for feeds of at most 32 tokens");
    if (b.len + t > b.cap) throw std::runtime_error("sequence exceeds the batch's max_len");
    int rows = 0;
    for (int c0 = 0; c0 < t; c0 += 32) {
        int len = std::min(32, t - c0);
        bool last = c0 + len >= t;
        int want = outputs;
        if ((outputs == ND_OUT_LAST_LOGITS || outputs == ND_OUT_LAST_HIDDEN) && !last) want = ND_OUT_NONE;
        const int32_t* src = dev_ids;
        if (t > 32) {
            // gather this chunk's columns [S][len] from ids [S][t]
            CK(cudaMemcpy2DAsync(b.ids, len * sizeof(int32_t), dev_ids + c0, t * sizeof(int32_t), len * sizeof(int32_t), b.S,
                                 cudaMemcpyDeviceToDevice, b.st));
            src = b.ids;
        }
        rows = chunk(b, src, len, want);
    }
    return rows;
}

// ----------------------------------------------------------- the C ABI

// After a synchronisation: the tensor-core prefill matmul records in a
// device word when one of its bounded waits expired (its results are then
// incomplete); report that as an error.
static void check_tc_waits() {
    const int e = tc_prefill_error();
    if (e > 0)
        throw std::runtime_error("tensor-core prefill matmul: a pipeline wait expired (stage " + std::to_string(e) +
                                 "); results of this call are incomplete");
}

static int fail(const std::exception& e) {
    g_err = e.what();
    return -1;
}

void set_error(const std::string& msg) { g_err = msg; }

}  // namespace nd

struct nd_model;

namespace nd {
bool model_head(const nd_model* m, DevMat* emb, int* device, int* out_rows);
bool model_embedding(const nd_model* m, DevMat* emb, int* device);
}  // namespace nd

using namespace nd;

struct nd_model {
    std::unique_ptr<Model> m;
};

// The tied lm_head matrix of a loaded model (for noalloc.cu).
bool nd::model_head(const nd_model* mh, DevMat* emb, int* device, int* out_rows) {
    if (!mh || !mh->m) return false;
    *emb = mh->m->head;
    *device = mh->m->device;
    *out_rows = mh->m->c.out_rows();
    return true;
}

// The whole token embedding of a loaded model, vocab rows (for ops.cu).
bool nd::model_embedding(const nd_model* mh, DevMat* emb, int* device) {
    if (!mh || !mh->m) return false;
    *emb = mh->m->embedding;
    *device = mh->m->device;
    return true;
}
struct nd_batch {
    std::unique_ptr<Batch> b;
    std::vector<int32_t> host_ids;
};

extern "C" {

const char* nd_last_error(void) { return g_err.c_str(); }

int nd_model_load(const unsigned char* cact, unsigned long long n, int device, nd_model** out) {
    try {
        if (!cact || !out) throw std::runtime_error("nd_model_load: null argument");
        nd_model* h = new nd_model();
        h->m.reset(load_model(cact, (size_t)n, device));
        *out = h;
        return 0;
    } catch (std::exception& e) {
        return fail(e);
    }
}

void nd_model_free(nd_model* m) { delete m; }

int nd_model_dims(const nd_model* mh, int* dims) {
    if (!mh || !dims) return -1;
    const Config& c = mh->m->c;
    int v[9] = {c.vocab, c.out_rows(), c.d, c.L, c.nh, c.nkv, c.qk, c.vd, c.max_seq};
    std::memcpy(dims, v, sizeof v);
    return 0;
}

int nd_batch_new(nd_model* mh, int num_seqs, int max_len, nd_batch** out) {
    try {
        if (!mh || !out) throw std::runtime_error("nd_batch_new: null argument");
        nd_batch* h = new nd_batch();
        h->b.reset(batch_new(mh->m.get(), num_seqs, max_len));
        *out = h;
        return 0;
    } catch (std::exception& e) {
        return fail(e);
    }
}

void nd_batch_free(nd_batch* b) { delete b; }

int nd_batch_len(const nd_batch* b) { return b ? b->b->len : -1; }

// The positions every sequence has been fed, on the host and the device.
static void set_len(Batch& b, int len) {
    b.len = len;
    CK(cudaMemcpyAsync(b.d_len, &b.len, sizeof(int32_t), cudaMemcpyHostToDevice, b.st));
    CK(cudaStreamSynchronize(b.st));
    b.have_logits = false;
}

int nd_batch_rollback(nd_batch* bh, int n) {
    try {
        if (!bh) throw std::runtime_error("nd_batch_rollback: null argument");
        Batch& b = *bh->b;
        CK(cudaSetDevice(b.m->device));
        if (n < 0 || n > 32) throw std::runtime_error("rollback of " + std::to_string(n) + " exceeds 32");
        if (n > b.len) throw std::runtime_error("rollback past the start of the sequence");
        if (n == 0) return 0;
        const int L = b.len - n;
        if (stale_below(b, L))
            throw std::runtime_error("the rollback leaves kept positions' ring slots to dropped ones (not served)");
        // infer.rs:1055-1077: the conv rows and engram history of positions
        // below L stay (the rings hold 32 positions more than a step reads),
        // as do the RoPE rows; a start before the conv history's start moves
        // it back, since the dropped positions are fed again
        b.hist_base = std::min(b.hist_base, L);
        b.rope_valid = L > 0 && L - 1 >= b.rope_from;
        set_len(b, L);
        return 0;
    } catch (std::exception& e) {
        return fail(e);
    }
}

int nd_batch_rewind_zeroed(nd_batch* bh, int len) {
    try {
        if (!bh) throw std::runtime_error("nd_batch_rewind_zeroed: null argument");
        Batch& b = *bh->b;
        CK(cudaSetDevice(b.m->device));
        if (len < 0 || len > b.len) throw std::runtime_error("rewind position outside [0, len]");
        if (stale_below(b, len))
            throw std::runtime_error("the rewind leaves kept positions' ring slots to dropped ones (not served)");
        // infer.rs:1039-1053: KV slots and slot map stay, the conv history
        // starts over (the next chunk reads zeros), the RoPE rows are dropped
        b.hist_base = len;
        b.rope_valid = false;
        b.rope_from = len;
        set_len(b, len);
        return 0;
    } catch (std::exception& e) {
        return fail(e);
    }
}

int nd_batch_truncate(nd_batch* bh, int len) {
    try {
        if (!bh) throw std::runtime_error("nd_batch_truncate: null argument");
        Batch& b = *bh->b;
        CK(cudaSetDevice(b.m->device));
        if (len < 0) throw std::runtime_error("truncate to a negative length");
        if (len >= b.len) return 0;
        if (b.len - len <= 32) {
            if (nd_batch_rollback(bh, b.len - len) != 0) throw std::runtime_error(g_err);
            return 0;
        }
        // model.rs:128-145: a fresh session (no attention span) fed the
        // first len tokens again
        int32_t* ids = nullptr;
        CK(cudaMallocAsync((void**)&ids, (size_t)b.S * std::max(len, 1) * sizeof(int32_t), b.st));
        if (len > 0)
            CK(cudaMemcpy2DAsync(ids, len * sizeof(int32_t), b.c.tokens, (size_t)b.cap * sizeof(int32_t), len * sizeof(int32_t), b.S,
                                 cudaMemcpyDeviceToDevice, b.st));
        if (nd_batch_set_attend(bh, 0, 0) != 0) throw std::runtime_error(g_err);
        b.slot_pos.clear();
        b.hist_base = 0;
        b.rope_valid = false;
        b.rope_from = 0;
        set_len(b, 0);
        if (len > 0) forward(b, ids, len, ND_OUT_NONE);
        CK(cudaFreeAsync(ids, b.st));
        CK(cudaStreamSynchronize(b.st));
        b.have_logits = false;
        return 0;
    } catch (std::exception& e) {
        return fail(e);
    }
}

int nd_batch_set_attend(nd_batch* bh, int sink, int ring) {
    try {
        if (!bh) throw std::runtime_error("nd_batch_set_attend: null argument");
        if (sink < 0 || ring < 0) throw std::runtime_error("nd_batch_set_attend: sink and ring must be non-negative");
        Batch& b = *bh->b;
        CK(cudaSetDevice(b.m->device));
        if (b.attend_sink == (ring > 0 ? sink : 0) && b.attend_ring == ring) return 0;
        // the captured decode steps bake the span into their launches
        CK(cudaStreamSynchronize(b.st));
        for (StepGraph& g : b.graph)
            if (g.exec) {
                cudaGraphExecDestroy(g.exec);
                g.exec = nullptr;
            }
        b.attend_sink = ring > 0 ? sink : 0;
        b.attend_ring = ring;
        return 0;
    } catch (std::exception& e) {
        return fail(e);
    }
}

void* nd_batch_stream(nd_batch* b) { return b ? (void*)b->b->st : nullptr; }

int nd_batch_forward(nd_batch* bh, const int* ids, int t, int outputs, float* out, int flags) {
    try {
        if (!bh || !ids) throw std::runtime_error("nd_batch_forward: null argument");
        Batch& b = *bh->b;
        CK(cudaSetDevice(b.m->device));
        const bool dev = flags & ND_DEVICE;
        const int32_t* dids = (const int32_t*)ids;
        int32_t* staging = nullptr;
        if (!dev) {
            CK(cudaMallocAsync((void**)&staging, (size_t)b.S * t * sizeof(int32_t), b.st));
            CK(cudaMemcpyAsync(staging, ids, (size_t)b.S * t * sizeof(int32_t), cudaMemcpyHostToDevice, b.st));
            dids = staging;
        }
        int rows = forward(b, dids, t, outputs);
        if (staging) CK(cudaFreeAsync(staging, b.st));
        if (out && outputs != ND_OUT_NONE) {
            const Config& c = b.m->c;
            size_t width = (outputs == ND_OUT_LAST_HIDDEN || outputs == ND_OUT_HIDDEN) ? c.d : c.out_rows();
            const float* src = width == (size_t)c.d ? b.h : b.logits;
            size_t n = (size_t)b.last_rows * width;
            CK(cudaMemcpyAsync(out, src, n * sizeof(float), dev ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost, b.st));
        }
        if (!dev) {
            CK(cudaStreamSynchronize(b.st));
            CK(cudaStreamSynchronize(b.st2));
            check_tc_waits();
        }
        return rows;
    } catch (std::exception& e) {
        return fail(e);
    }
}

int nd_batch_step(nd_batch* bh, const unsigned char* allow_bits, int* next_ids, int flags) {
    try {
        if (!bh) throw std::runtime_error("nd_batch_step: null argument");
        Batch& b = *bh->b;
        CK(cudaSetDevice(b.m->device));
        if (!b.have_logits || b.logits_rows != b.S) throw std::runtime_error("nd_batch_step needs the last logits of every sequence");
        const bool dev = flags & ND_DEVICE;
        const Config& c = b.m->c;
        const size_t mb = (size_t)(c.out_rows() + 7) / 8;
        const uint8_t* allow = allow_bits;
        if (allow_bits && !dev) {
            CK(cudaMemcpyAsync(b.masks, allow_bits, (size_t)b.S * mb, cudaMemcpyHostToDevice, b.st));
            allow = b.masks;
        }
        if (allow_bits && dev) {
            CK(cudaMemcpyAsync(b.masks, allow_bits, (size_t)b.S * mb, cudaMemcpyDeviceToDevice, b.st));
            allow = b.masks;
        }
        // The step (argmax, then one decode forward) replays as a CUDA graph
        // once captured: every kernel reads its position on the device.
        const bool graph_ok = b.graphs && b.rope_valid && b.debug_layer < 0 && b.time_site == 0;
        if (graph_ok) {
            StepGraph& g = b.graph[allow ? 1 : 0];
            if (g.exec && g.hist_base != b.hist_base) {
                cudaGraphExecDestroy(g.exec);
                g.exec = nullptr;
            }
            if (!g.exec) {
                const long long k0 = launch_count();
                cudaGraph_t graph = nullptr;
                CK(cudaStreamBeginCapture(b.st, cudaStreamCaptureModeThreadLocal));
                try {
                    launch_masked_argmax(b.logits, b.S, c.out_rows(), allow, b.next, b.st);
                    forward(b, b.next, 1, ND_OUT_LAST_LOGITS);  // advances the host state once
                } catch (...) {
                    cudaStreamEndCapture(b.st, &graph);
                    if (graph) cudaGraphDestroy(graph);
                    throw;
                }
                CK(cudaStreamEndCapture(b.st, &graph));
                cudaError_t ie = cudaGraphInstantiate(&g.exec, graph, 0);
                cudaGraphDestroy(graph);
                CK(ie);
                g.kernels = launch_count() - k0;
                g.hist_base = b.hist_base;
                CK(cudaGraphLaunch(g.exec, b.st));
            } else {
                CK(cudaGraphLaunch(g.exec, b.st));
                add_launches(g.kernels);
                mark_slots(b, b.len, 1);
                b.len += 1;
                b.last_T = 1;
                b.last_rows = b.S;
                b.have_logits = true;
                b.logits_rows = b.S;
            }
        } else {
            // with a site timed, queue the whole step behind a 5 ms hold
            if (b.time_site) launch_hold(5000000ull, b.st);
            launch_masked_argmax(b.logits, b.S, c.out_rows(), allow, b.next, b.st);
            forward(b, b.next, 1, ND_OUT_LAST_LOGITS);
        }
        if (next_ids)
            CK(cudaMemcpyAsync(next_ids, b.next, (size_t)b.S * sizeof(int32_t),
                               dev ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost, b.st));
        if (!dev) CK(cudaStreamSynchronize(b.st));
        return 0;
    } catch (std::exception& e) {
        return fail(e);
    }
}

int nd_batch_last_hidden(nd_batch* bh, float* out, int flags) {
    try {
        Batch& b = *bh->b;
        CK(cudaSetDevice(b.m->device));
        if (b.last_rows < 1) throw std::runtime_error("no forward has returned outputs yet");
        // the last row of each sequence's outputs
        const int per = b.last_rows / b.S;
        CK(cudaMemcpy2DAsync(out, 768 * sizeof(float), b.h + (size_t)(per - 1) * 768, (size_t)per * 768 * sizeof(float),
                             768 * sizeof(float), b.S, (flags & ND_DEVICE) ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost,
                             b.st));
        if (!(flags & ND_DEVICE)) CK(cudaStreamSynchronize(b.st));
        return 0;
    } catch (std::exception& e) {
        return fail(e);
    }
}

int nd_head_logits(nd_batch* bh, const float* h, int rows, float* out, int flags) {
    try {
        Batch& b = *bh->b;
        Model& m = *b.m;
        CK(cudaSetDevice(m.device));
        if (rows < 1 || rows > b.Mmax) throw std::runtime_error("nd_head_logits: rows out of range");
        const bool dev = flags & ND_DEVICE;
        CK(cudaMemcpyAsync(b.e, h, (size_t)rows * 768 * sizeof(float), dev ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice,
                           b.st));
        ensure_logits(b, rows);
        launch_prep_act(b.e, 768, 768, rows, b.act, b.sx, b.st);
        CK(launch_cq_gemm(m.head, b.act, b.sx, rows, 1, b.logits, m.c.out_rows(), 0, b.st));
        b.have_logits = false;
        CK(cudaMemcpyAsync(out, b.logits, (size_t)rows * m.c.out_rows() * sizeof(float),
                           dev ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost, b.st));
        if (!dev) CK(cudaStreamSynchronize(b.st));
        return 0;
    } catch (std::exception& e) {
        return fail(e);
    }
}

int nd_head_logits_sparse(nd_batch* bh, const float* h, const int* ids, int n, float* out) {
    try {
        Batch& b = *bh->b;
        Model& m = *b.m;
        const int V = m.c.out_rows();
        for (int k = 0; k < n; k++)
            if (ids[k] < 0 || ids[k] >= V) throw std::runtime_error("nd_head_logits_sparse: id out of range");
        // the single-row kernel is the prefill combine's block form
        // (qlinear.rs:454-456): each id scored as a lone block token, i.e.
        // a T = 4 feed of which it is row 0.
        CK(cudaSetDevice(m.device));
        std::vector<float> h4(4 * 768, 0.f);
        std::memcpy(h4.data(), h, 768 * sizeof(float));
        CK(cudaMemcpyAsync(b.e, h4.data(), 4 * 768 * sizeof(float), cudaMemcpyHostToDevice, b.st));
        ensure_logits(b, 4);
        launch_prep_act(b.e, 768, 768, 4, b.act, b.sx, b.st);
        CK(launch_cq_gemm(m.head, b.act, b.sx, 4, 4, b.logits, V, 0, b.st));
        b.have_logits = false;
        std::vector<float> full(V);
        CK(cudaMemcpyAsync(full.data(), b.logits, V * sizeof(float), cudaMemcpyDeviceToHost, b.st));
        CK(cudaStreamSynchronize(b.st));
        uint32_t negu = 0xf149f2cau;
        float neg;
        std::memcpy(&neg, &negu, 4);
        for (int k = 0; k < V; k++) out[k] = neg;
        for (int k = 0; k < n; k++) out[ids[k]] = full[ids[k]];
        return 0;
    } catch (std::exception& e) {
        return fail(e);
    }
}

int nd_batch_candidates(nd_batch* bh, const float* logits, const unsigned char* allow, const unsigned char* allow_order, int k,
                        int* ids, float* m, double* z, int* live, int flags) {
    try {
        if (!bh || !ids || !m || !z || !live) throw std::runtime_error("nd_batch_candidates: null argument");
        Batch& b = *bh->b;
        CK(cudaSetDevice(b.m->device));
        if (!logits && (!b.have_logits || b.logits_rows != b.S))
            throw std::runtime_error("nd_batch_candidates needs the last logits of every sequence");
        if (k < 1 || k > 128) throw std::runtime_error("nd_batch_candidates: k must be in [1, 128]");
        const int V = b.m->c.out_rows();
        if (V > 65536) throw std::runtime_error("nd_batch_candidates: more than 65536 logits a row");
        const bool dev = flags & ND_DEVICE;
        const size_t mb = (size_t)(V + 7) / 8;
        if (!b.cids) {
            b.clogits = b.alloc<float>((size_t)b.S * V);
            b.cex = b.alloc<float>((size_t)b.S * V);
            b.cmask1 = b.alloc<uint8_t>((size_t)b.S * mb);
            b.cmask2 = b.alloc<uint8_t>((size_t)b.S * mb);
            b.cids = b.alloc<int32_t>((size_t)b.S * 128);
            b.clive = b.alloc<int32_t>((size_t)b.S);
            b.cm = b.alloc<float>((size_t)b.S);
            b.cz = b.alloc<double>((size_t)b.S);
        }
        const float* src = b.logits;
        if (logits && dev) src = logits;
        if (logits && !dev) {
            CK(cudaMemcpyAsync(b.clogits, logits, (size_t)b.S * V * sizeof(float), cudaMemcpyHostToDevice, b.st));
            src = b.clogits;
        }
        const uint8_t *a1 = allow, *a2 = allow_order;
        if (allow && !dev) {
            CK(cudaMemcpyAsync(b.cmask1, allow, (size_t)b.S * mb, cudaMemcpyHostToDevice, b.st));
            a1 = b.cmask1;
        }
        if (allow_order && !dev) {
            CK(cudaMemcpyAsync(b.cmask2, allow_order, (size_t)b.S * mb, cudaMemcpyHostToDevice, b.st));
            a2 = b.cmask2;
        }
        int32_t* di = dev ? (int32_t*)ids : b.cids;
        int32_t* dl = dev ? (int32_t*)live : b.clive;
        float* dm = dev ? m : b.cm;
        double* dz = dev ? z : b.cz;
        CK(launch_candidates(src, b.S, V, a1, a2, k, di, dm, dz, dl, b.cex, b.st));
        if (!dev) {
            CK(cudaMemcpyAsync(ids, b.cids, (size_t)b.S * k * sizeof(int32_t), cudaMemcpyDeviceToHost, b.st));
            CK(cudaMemcpyAsync(live, b.clive, (size_t)b.S * sizeof(int32_t), cudaMemcpyDeviceToHost, b.st));
            CK(cudaMemcpyAsync(m, b.cm, (size_t)b.S * sizeof(float), cudaMemcpyDeviceToHost, b.st));
            CK(cudaMemcpyAsync(z, b.cz, (size_t)b.S * sizeof(double), cudaMemcpyDeviceToHost, b.st));
            CK(cudaStreamSynchronize(b.st));
        }
        return 0;
    } catch (std::exception& e) {
        return fail(e);
    }
}

// heads.rs:63-66 for every sequence of a fresh batch: ids [S][T] fed in
// chunks of 32 with the cells of every position and depth recorded, then
// head h's pool (kind as launch_probe_head) into b.head_out [S][width].
static void probe_run(Batch& b, const int* ids, int T, int flags, const HeadW& h, int kind, int width) {
    const Config& c = b.m->c;
    if (b.len != 0) throw std::runtime_error("the probe heads read a fresh batch (no position fed yet)");
    if (T < 1 || T > b.cap) throw std::runtime_error("token count outside [1, max_len]");
    const int l1 = c.L + 1;
    if (b.cells_cap < T) {
        b.cells = b.alloc<float>((size_t)b.S * T * l1 * c.d);
        b.cells_cap = T;
    }
    if (!b.head_r) {
        // every head here has k <= 16 probes a depth and q <= 16 queries
        b.head_r = b.alloc<float>((size_t)b.S * l1 * 16 * c.d);
        b.head_pool = b.alloc<float>((size_t)b.S * 16 * c.d);
        b.head_out = b.alloc<float>((size_t)b.S * 16 * c.d);
    }
    if (h.k > 16 || h.q > 16 || width > 16 * c.d) throw std::runtime_error("probe head larger than this engine serves");
    const bool dev = flags & ND_DEVICE;
    const int32_t* dids = (const int32_t*)ids;
    int32_t* staging = nullptr;
    if (!dev) {
        CK(cudaMallocAsync((void**)&staging, (size_t)b.S * T * sizeof(int32_t), b.st));
        CK(cudaMemcpyAsync(staging, ids, (size_t)b.S * T * sizeof(int32_t), cudaMemcpyHostToDevice, b.st));
        dids = staging;
    }
    b.recording = true;
    try {
        forward(b, dids, T, ND_OUT_NONE);
    } catch (...) {
        b.recording = false;
        throw;
    }
    b.recording = false;
    if (staging) CK(cudaFreeAsync(staging, b.st));
    launch_probe_head(h, b.cells, b.S, T, b.cells_cap, l1, kind, b.head_r, b.head_pool, b.head_out, b.st);
    CK(cudaGetLastError());
}

int nd_batch_embed(nd_batch* bh, const int* ids, int T, float* out, int* dim, int flags) {
    try {
        if (!bh) throw std::runtime_error("nd_batch_embed: null argument");
        Batch& b = *bh->b;
        Model& m = *b.m;
        CK(cudaSetDevice(m.device));
        // heads.rs:80-84: the embedding head, else the confidence head's pool
        int kind, width;
        const HeadW* h;
        if (m.has_head[0]) {
            h = &m.heads[0];
            kind = 0;
            width = h->out;
        } else if (m.has_head[1]) {
            h = &m.heads[1];
            kind = 1;
            width = h->q * m.c.d;
        } else {
            throw std::runtime_error("this archive carries no probe head");
        }
        if (dim) *dim = width;
        if (!out) return 0;
        if (!ids) throw std::runtime_error("nd_batch_embed: null ids");
        probe_run(b, ids, T, flags, *h, kind, width);
        const bool dev = flags & ND_DEVICE;
        CK(cudaMemcpyAsync(out, b.head_out, (size_t)b.S * width * sizeof(float),
                           dev ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost, b.st));
        if (!dev) CK(cudaStreamSynchronize(b.st));
        return 0;
    } catch (std::exception& e) {
        return fail(e);
    }
}

int nd_batch_confidence(nd_batch* bh, const int* ids, int T, float* out, int flags) {
    try {
        if (!bh || !ids || !out) throw std::runtime_error("nd_batch_confidence: null argument");
        Batch& b = *bh->b;
        Model& m = *b.m;
        CK(cudaSetDevice(m.device));
        if (!m.has_head[1]) throw std::runtime_error("this archive carries no confidence head");
        probe_run(b, ids, T, flags, m.heads[1], 2, 1);
        const bool dev = flags & ND_DEVICE;
        CK(cudaMemcpyAsync(out, b.head_out, (size_t)b.S * sizeof(float), dev ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost,
                           b.st));
        if (!dev) CK(cudaStreamSynchronize(b.st));
        return 0;
    } catch (std::exception& e) {
        return fail(e);
    }
}

// One CQ matrix on a GPU for kernel-level tests and the matmul sweep.
struct nd_cqmat {
    Model m;  // owns the uploads
    DevMat d;
    cudaStream_t st = nullptr;
    float *x = nullptr, *y = nullptr, *sx = nullptr;
    int8_t* act = nullptr;
    int cap = 0;
    std::vector<void*> scratch;
    ~nd_cqmat() {
        cudaSetDevice(m.device);
        if (st) cudaStreamSynchronize(st);
        for (void* p : scratch) cudaFree(p);
        if (st) cudaStreamDestroy(st);
    }
};

int nd_cqmat_new(int device, const unsigned char* codes, const unsigned short* norms, int out, int in_dim, int bits,
                 nd_cqmat** h) {
    try {
        if (!codes || !norms || !h) throw std::runtime_error("nd_cqmat_new: null argument");
        if (in_dim != 768) throw std::runtime_error("nd_cqmat_new: the engine's matmuls take in_dim 768");
        if (out < 1) throw std::runtime_error("nd_cqmat_new: out must be positive");
        const int width = cq_width(bits);
        CK(cudaSetDevice(device));
        std::unique_ptr<nd_cqmat> q(new nd_cqmat());
        q->m.device = device;
        HostMat hm;
        hm.out = out;
        hm.in_dim = in_dim;
        hm.groups = 6;
        hm.bits = bits;
        hm.codes.assign(codes, codes + (size_t)out * 6 * 16 * width);
        hm.norms.assign(norms, norms + (size_t)out * 6);
        q->d = to_dev(q->m, hm, true);
        set_constants((float)(1.0 / std::sqrt(128.0)));
        CK(cudaGetLastError());
        CK(cudaStreamCreateWithFlags(&q->st, cudaStreamNonBlocking));
        *h = q.release();
        return 0;
    } catch (std::exception& e) {
        return fail(e);
    }
}

void nd_cqmat_free(nd_cqmat* h) { delete h; }

int nd_cqmat_apply(nd_cqmat* h, const float* x, int M, int T, float* y, int reps, float* ms) {
    try {
        if (!h || !x || !y) throw std::runtime_error("nd_cqmat_apply: null argument");
        if (M < 1 || T < 1 || M % T) throw std::runtime_error("nd_cqmat_apply: M must be a positive multiple of T");
        CK(cudaSetDevice(h->m.device));
        const int out = h->d.out;
        if (M > h->cap) {
            for (void* p : h->scratch) cudaFree(p);
            h->scratch.clear();
            auto get = [&](size_t bytes) {
                void* p = nullptr;
                CK(cudaMalloc(&p, bytes + 64));
                h->scratch.push_back(p);
                return p;
            };
            h->x = (float*)get((size_t)M * 768 * 4);
            h->act = (int8_t*)get((size_t)M * 768);
            h->sx = (float*)get((size_t)M * 8 * 4);
            h->y = (float*)get((size_t)M * out * 4);
            h->cap = M;
        }
        CK(cudaMemcpyAsync(h->x, x, (size_t)M * 768 * 4, cudaMemcpyHostToDevice, h->st));
        auto run = [&]() {
            launch_prep_act(h->x, 768, 768, M, h->act, h->sx, h->st);
            CK(launch_cq_gemm(h->d, h->act, h->sx, M, T, h->y, out, 0, h->st));
        };
        run();
        if (reps > 0 && ms) {
            cudaEvent_t e0, e1;
            CK(cudaEventCreate(&e0));
            CK(cudaEventCreate(&e1));
            for (int k = 0; k < 3; k++) run();
            CK(cudaEventRecord(e0, h->st));
            for (int k = 0; k < reps; k++) run();
            CK(cudaEventRecord(e1, h->st));
            CK(cudaEventSynchronize(e1));
            float t = 0;
            CK(cudaEventElapsedTime(&t, e0, e1));
            *ms = t / reps;
            cudaEventDestroy(e0);
            cudaEventDestroy(e1);
        }
        CK(cudaGetLastError());
        CK(cudaMemcpyAsync(y, h->y, (size_t)M * out * 4, cudaMemcpyDeviceToHost, h->st));
        CK(cudaStreamSynchronize(h->st));
        check_tc_waits();
        return 0;
    } catch (std::exception& e) {
        return fail(e);
    }
}

int nd_cqmat_time_rotating(nd_cqmat* const* mats, int n, int M, int T, int reps, float* ms) {
    try {
        if (!mats || n < 1 || !ms || reps < 1) throw std::runtime_error("nd_cqmat_time_rotating: bad arguments");
        nd_cqmat* h = mats[0];
        if (!h || M < 1 || T < 1 || M % T || M > h->cap)
            throw std::runtime_error("nd_cqmat_time_rotating: M must be a multiple of T within the last apply's rows");
        for (int i = 0; i < n; i++)
            if (!mats[i] || mats[i]->m.device != h->m.device || mats[i]->d.out != h->d.out)
                throw std::runtime_error("nd_cqmat_time_rotating: matrices must share the device and shape");
        CK(cudaSetDevice(h->m.device));
        const int out = h->d.out;
        auto round = [&]() {
            for (int i = 0; i < n; i++) CK(launch_cq_gemm(mats[i]->d, h->act, h->sx, M, T, h->y, out, 0, h->st));
        };
        cudaEvent_t e0, e1;
        CK(cudaEventCreate(&e0));
        CK(cudaEventCreate(&e1));
        round();
        CK(cudaEventRecord(e0, h->st));
        for (int k = 0; k < reps; k++) round();
        CK(cudaEventRecord(e1, h->st));
        CK(cudaEventSynchronize(e1));
        float t = 0;
        CK(cudaEventElapsedTime(&t, e0, e1));
        *ms = t / ((float)reps * n);
        cudaEventDestroy(e0);
        cudaEventDestroy(e1);
        CK(cudaGetLastError());
        return 0;
    } catch (std::exception& e) {
        return fail(e);
    }
}

int nd_cq_pack(const float* w, int rows, int d, int bits, unsigned char* codes, unsigned short* norms) {
    try {
        cq_pack(w, rows, d, bits, codes, norms);
        return 0;
    } catch (std::exception& e) {
        return fail(e);
    }
}

int nd_synth_cact(int num_layers, int vocab, int engram_slots, int sliding_window, unsigned long long global_mask,
                  unsigned long long engram_sites, unsigned long long seed, float std, const int* cq_bits, int n_cq_bits,
                  unsigned heads_mask, unsigned char* out, unsigned long long cap, unsigned long long* len) {
    try {
        SynthSpec sp;
        if (heads_mask & ~0xEu) throw std::runtime_error("nd_synth_cact: probe head codes are 1, 2 and 3");
        sp.heads_mask = heads_mask;
        if (n_cq_bits < 0 || (n_cq_bits > 0 && !cq_bits)) throw std::runtime_error("nd_synth_cact: bad code width list");
        sp.cq_bits.assign(cq_bits, cq_bits + n_cq_bits);
        sp.num_layers = num_layers;
        sp.vocab = vocab;
        sp.engram_slots = engram_slots;
        sp.sliding_window = sliding_window;
        sp.global_mask = global_mask;
        sp.engram_sites.clear();
        for (int l = 0; l < 64; l++)
            if ((engram_sites >> l) & 1) sp.engram_sites.push_back(l);
        sp.seed = seed;
        sp.std = std;
        std::vector<uint8_t> buf = synth_cact(sp);
        if (len) *len = buf.size();
        if (out) {
            if (cap < buf.size()) throw std::runtime_error("nd_synth_cact: buffer too small");
            std::memcpy(out, buf.data(), buf.size());
        }
        return 0;
    } catch (std::exception& e) {
        return fail(e);
    }
}

long long nd_launch_count(void) { return launch_count(); }

int nd_batch_time_site(nd_batch* bh, int site) {
    if (!bh) return -1;
    Batch& b = *bh->b;
    b.time_site = site;
    b.ev_used = 0;
    return 0;
}

int nd_batch_site_time(nd_batch* bh, double* total_ms, int* launches) {
    try {
        Batch& b = *bh->b;
        CK(cudaSetDevice(b.m->device));
        CK(cudaStreamSynchronize(b.st));
        double tot = 0;
        for (size_t k = 0; k + 1 < b.ev_used; k += 2) {
            float ms = 0;
            CK(cudaEventElapsedTime(&ms, b.evs[k], b.evs[k + 1]));
            tot += ms;
        }
        if (total_ms) *total_ms = tot;
        if (launches) *launches = (int)(b.ev_used / 2);
        return 0;
    } catch (std::exception& e) {
        return fail(e);
    }
}

int nd_batch_debug_layer(nd_batch* bh, int layer) {
    if (!bh) return -1;
    bh->b->debug_layer = layer;
    return 0;
}

int nd_batch_debug(nd_batch* bh, const char* name, float* out, long long cap) {
    try {
        Batch& b = *bh->b;
        CK(cudaSetDevice(b.m->device));
        CK(cudaStreamSynchronize(b.st));
        const int M = b.S * b.last_T;
        std::string nm(name);
        const float* src = nullptr;
        size_t n = 0;
        if (nm.rfind("snap.", 0) == 0) {
            auto it = b.snaps.find(nm);
            if (it == b.snaps.end()) return -1;
            src = it->second.first;
            n = it->second.second;
        } else if (nm == "xs") { src = b.xs; n = (size_t)M * 3072; }
        else if (nm == "u") { src = b.u; n = (size_t)M * 768; }
        else if (nm == "p") { src = b.p; n = (size_t)M * 24; }
        else if (nm == "x1") { src = b.x1; n = (size_t)M * 768; }
        else if (nm == "proj") { src = b.proj; n = (size_t)M * 1568; }
        else if (nm == "qbuf") { src = b.qbuf; n = (size_t)M * 576; }
        else if (nm == "att") { src = b.att; n = (size_t)M * 768; }
        else if (nm == "o") { src = b.o; n = (size_t)M * 768; }
        else if (nm == "h") { src = b.h; n = (size_t)b.last_rows * 768; }
        else if (nm == "logits") { src = b.logits; n = b.logits ? (size_t)b.logits_rows * b.m->c.out_rows() : 0; }
        else if (nm.rfind("ekv", 0) == 0) { src = b.ekv + (size_t)std::stoi(nm.substr(3)) * b.Mmax * 1536; n = (size_t)M * 1536; }
        else if (nm.rfind("evals", 0) == 0) { src = b.evals + (size_t)std::stoi(nm.substr(5)) * b.Mmax * 768; n = (size_t)M * 768; }
        else return -1;
        if (!src) return -1;
        if (out) CK(cudaMemcpy(out, src, std::min<size_t>(n, (size_t)cap) * sizeof(float), cudaMemcpyDeviceToHost));
        return (int)n;
    } catch (std::exception& e) {
        return fail(e);
    }
}

// ------------------------------------------------------------- needle.h

static std::mutex g_engine_mu;
static std::unique_ptr<nd_model> g_model;
static std::string g_needle_err;

static int needle_fail(const std::string& msg, int code) {
    g_needle_err = msg;
    return code;
}

int needle_load(const unsigned char* cact, unsigned long long n) {
    std::lock_guard<std::mutex> lk(g_engine_mu);
    if (!cact) return needle_fail("needle_load: null archive", -1);
    int device = 0;
    if (const char* d = getenv("NEEDLE_DEVICE")) device = atoi(d);
    nd_model* m = nullptr;
    if (nd_model_load(cact, n, device, &m) != 0) return needle_fail(g_err, -1);
    g_model.reset(m);
    return 0;
}

static const char* AGENT_MISSING =
    "the agent layer (tokenizer, chat template, tool-call grammar) is not part of this GPU engine; drive the model "
    "through needle_engine.h";

int needle_init(const char*, const char*, const char*) {
    std::lock_guard<std::mutex> lk(g_engine_mu);
    if (!g_model) return needle_fail("no model loaded: call needle_load first", -1);
    return needle_fail(AGENT_MISSING, -1);
}

int needle_complete(const char*, int, char* out, int out_capacity) {
    std::lock_guard<std::mutex> lk(g_engine_mu);
    std::string msg = "no toolset bound: call needle_init first";
    g_needle_err = msg;
    if (out && out_capacity > (int)msg.size()) {
        std::memcpy(out, msg.c_str(), msg.size() + 1);
    }
    return -1;
}

int needle_embed(const char*, float* out, int) {
    std::lock_guard<std::mutex> lk(g_engine_mu);
    if (!g_model) return needle_fail("no model loaded", -1);
    // lib.rs:152: confidence_queries * d_model when the archive has no
    // embedding head (probe heads are not loaded by this engine).
    if (!out) return 4 * g_model->m->c.d;
    return needle_fail("no toolset bound: call needle_init first", -1);
}

void needle_reset(void) {}

const char* needle_last_error(void) { return g_needle_err.c_str(); }

}  // extern "C"
