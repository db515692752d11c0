// TEST INFRASTRUCTURE ONLY — never linked into or called by the product path.
//
// A C++ restatement of ddrscott/needle-rs's packed CPU inference path (the
// native-exact `needle-engine` forward pass on a `.cact` archive), used by
// tests/ as the parity checker for the CUDA engine and by bench.py as the
// timed CPU baseline ("port"). The reference is Rust and cannot be built in
// this image (no cargo/rustc), so this file restates its arithmetic from the
// source. Every function names the reference file:line it follows; paths are
// relative to the needle-rs repository root. The spec is the portable scalar
// branch of each reference function (the `#[cfg(not(aarch64|wasm32))]` arms
// and the `*_ref` functions the SIMD kernels are tested bit-equal against).
//
// Float discipline: compiled with -ffp-contract=off; every `mul_add` of the
// reference is an explicit fmaf here, every other op is a single IEEE op in
// the reference's order. Integer sums are exact and computed in any order.
// Where the build has AVX2 the hot loops run vectorised without changing a
// result: the int8 lane sums and dots (4-bit codes looked up from their
// packed bytes; byte pair products into int16 only when no operand is -128,
// else int16 pair products into int32, or AVX-512 VNNI byte products into
// int32 where the host has it: nothing saturates; attention's P·V sums
// likewise on VNNI), the decode combine eight rows side by side, the
// Kronecker passes eight outputs side by side, the inline exp and the int8
// quantizer eight values at a time (each row's, output's or value's float
// ops the same single roundings in the same order). orc_lane_sums_check,
// orc_nexp_check, orc_quant_check and orc_pv_check compare the vector forms
// with the plain loops.
// libm stand-ins follow the reference's non-Apple `sys` module
// (crates/needle-engine/src/infer.rs:83-102): f32 exp/pow/sincos are f64 libm
// rounded once; this file uses glibc's f64 functions where the reference links
// the `libm` crate 0.2.16 (parity of those last bits is not pinned).

#include <cmath>
#include <cstdint>
#include <cstring>
#include <cstdlib>
#include <cstdio>
#include <string>
#include <vector>
#include <map>
#include <thread>
#include <atomic>
#include <algorithm>
#include <functional>
#include <stdexcept>
#include <mutex>
#include <condition_variable>
#include <exception>
#if defined(__AVX2__)
#include <immintrin.h>
#endif

namespace orc {

// ---------------------------------------------------------------- the team

// What the reference's worker team (crates/needle-engine/src/team.rs) does
// for one sequence: the rows of a matmul, the heads of attention and the
// rows of a chunk's post block split over host threads. Every item is
// computed by one thread exactly as the single-threaded loop computes it,
// so results do not depend on the team's size. One thread (no team) unless
// orc_set_team asks for more; the threads of a sequence-parallel batch
// (run_parallel) never use it.
thread_local bool t_no_team = false;

class Team {
public:
    ~Team() { resize(1); }
    int size() const { return (int)workers_.size() + 1; }
    void resize(int n) {
        stop_.store(true);
        gen_.fetch_add(1);
        {
            std::lock_guard<std::mutex> lk(mu_);
            cv_.notify_all();
        }
        for (auto& w : workers_) w.join();
        workers_.clear();
        stop_.store(false);
        // each worker starts from the counter as it is now, read here: a
        // job published before a new thread first runs is still its job
        const uint64_t start = gen_.load();
        for (int k = 1; k < n; k++) workers_.emplace_back([this, start] { loop(start); });
    }
    // f(i0, i1) over contiguous slices of [0, items), the calling thread
    // taking slices too; returns when every slice is done, then rethrows
    // the first exception a slice threw (the other slices still ran).
    void run(int items, const std::function<void(int, int)>& f) {
        if (items <= 0) return;
        if (workers_.empty() || t_no_team || items == 1) {
            f(0, items);
            return;
        }
        job_ = &f;
        items_ = items;
        slices_ = std::min(items, 4 * size());
        next_.store(0);
        busy_.store((int)workers_.size());
        gen_.fetch_add(1);  // publishes the job (sequentially consistent)
        if (sleeping_.load() > 0) {
            std::lock_guard<std::mutex> lk(mu_);
            cv_.notify_all();
        }
        work();
        while (busy_.load() != 0) pause();
        job_ = nullptr;
        if (error_) {
            std::exception_ptr e = error_;
            error_ = nullptr;
            std::rethrow_exception(e);
        }
    }

private:
    static void pause() {
#if defined(__x86_64__)
        __builtin_ia32_pause();
#endif
    }
    void work() {
        for (;;) {
            const int k = next_.fetch_add(1);
            if (k >= slices_) return;
            try {
                (*job_)((int)((int64_t)items_ * k / slices_), (int)((int64_t)items_ * (k + 1) / slices_));
            } catch (...) {
                std::lock_guard<std::mutex> lk(err_mu_);
                if (!error_) error_ = std::current_exception();
            }
        }
    }
    // A worker spins on the job counter for a while after each job (a
    // sequence's parallel regions come tens of microseconds apart), then
    // sleeps; a sleeper counts itself before it tests the counter, and run()
    // bumps the counter before it reads the sleepers, so one of the two
    // always sees the other.
    void loop(uint64_t seen) {
        t_no_team = true;
        for (;;) {
            int spins = 0;
            while (gen_.load() == seen && spins < (1 << 16)) {
                pause();
                spins++;
            }
            if (gen_.load() == seen) {
                std::unique_lock<std::mutex> lk(mu_);
                sleeping_.fetch_add(1);
                cv_.wait(lk, [&] { return gen_.load() != seen; });
                sleeping_.fetch_sub(1);
            }
            seen = gen_.load();
            if (stop_.load()) return;
            work();
            busy_.fetch_sub(1);
        }
    }
    std::vector<std::thread> workers_;
    std::mutex mu_, err_mu_;
    std::exception_ptr error_;
    std::condition_variable cv_;
    const std::function<void(int, int)>* job_ = nullptr;
    int items_ = 0, slices_ = 0;
    std::atomic<int> next_{0}, busy_{0}, sleeping_{0};
    std::atomic<uint64_t> gen_{0};
    std::atomic<bool> stop_{false};
};

static Team g_team;

// AVX-512 VNNI on this host (the 4-bit lane sums and attention's P·V sums
// use it where present; ORC_NO_VNNI in the environment turns it off).
static bool vnni_host() {
#if defined(__AVX2__) && defined(__x86_64__)
    static const bool v = __builtin_cpu_supports("avx512f") && __builtin_cpu_supports("avx512bw") &&
                          __builtin_cpu_supports("avx512vl") && __builtin_cpu_supports("avx512vnni") &&
                          !std::getenv("ORC_NO_VNNI");
    return v;
#else
    return false;
#endif
}

// ---------------------------------------------------------------- numerics

static inline uint32_t fbits(float f) { uint32_t u; std::memcpy(&u, &f, 4); return u; }
static inline float bitsf(uint32_t u) { float f; std::memcpy(&f, &u, 4); return f; }

// `half` 2.7.1 f16 <-> f32, round to nearest even (Cargo.lock pins half 2.7.1).
float f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1f, m = h & 0x3ff;
    if (e == 0) {
        float v = (float)m * 5.9604644775390625e-8f;  // m * 2^-24, exact
        return bitsf(fbits(v) | sign);
    }
    if (e == 31) return bitsf(sign | 0x7f800000u | (m << 13));
    return bitsf(sign | ((e + 112) << 23) | (m << 13));
}

uint16_t f32_to_f16(float f) {
    uint32_t x = fbits(f);
    uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
    uint32_t ax = x & 0x7fffffffu;
    if (ax >= 0x7f800000u) return sign | (ax > 0x7f800000u ? 0x7e00 : 0x7c00);
    if (ax >= 0x477ff000u) return sign | 0x7c00;
    if (ax < 0x38800000u) {
        float s = bitsf(ax) * 16777216.0f;  // exact power-of-two scaling
        return sign | (uint16_t)std::nearbyint(s);
    }
    uint32_t h = (((ax >> 23) - 112) << 10) | ((ax & 0x7fffff) >> 13);
    uint32_t rem = ax & 0x1fff;
    if (rem > 0x1000 || (rem == 0x1000 && (h & 1))) h++;
    return sign | (uint16_t)h;
}

// crates/needle-engine/src/infer.rs:83-102 (non-Apple `sys`).
static inline float lexpf(float x) { return (float)std::exp((double)x); }
static inline double lexp(double x) { return std::exp(x); }
static inline float lpowf(float x, float y) { return (float)std::pow((double)x, (double)y); }
static inline void lsincosf(float x, float* s, float* c) {
    double sd, cd;
    sincos((double)x, &sd, &cd);
    *s = (float)sd;
    *c = (float)cd;
}

// crates/needle-engine/src/qlinear.rs:40
static const float K127 = bitsf(0x3c010204u);
// crates/needle-engine/src/infer.rs:30-36
static const float INV_SQRT_QK = bitsf(0x3e13cd3au);
static const float Q21 = bitsf(0x49fffff8u);
static const float C21 = bitsf(0x35000004u);
static const float NEG = bitsf(0xf149f2cau);
static const int NATIVE_TEAM = 4;  // infer.rs:38
static const int ROLLBACK = 32;    // model.rs:184
static const int GROUP = 128;      // qlinear.rs:37

// Rust f32::max / f32::min (IEEE maxNum: a NaN operand loses).
static inline float rmax(float a, float b) { return std::fmax(a, b); }
static inline float rmin(float a, float b) { return std::fmin(a, b); }
// Rust f32::round: half away from zero.
static inline float rround(float x) { return std::round(x); }

// f32::max as the reference's platform computes it (aarch64 FMAXNM: -0 < +0).
static inline float fmaxnm(float a, float b) {
    if (a > b) return a;
    if (b > a) return b;
    return std::signbit(a) ? b : a;
}


// crates/needle-engine/src/infer.rs:353-366
float nexp(float x) {
    x = rmin(rmax(x, bitsf(0xc2b0c0a5u)), bitsf(0x42b0c0a5u));
    float k = std::nearbyint(x * bitsf(0x3fb8aa3bu));  // round_ties_even
    float r = std::fmaf(k, bitsf(0xbf318000u), x);
    r = std::fmaf(k, bitsf(0x395e8083u), r);
    float p = std::fmaf(bitsf(0x39506967u), r, bitsf(0x3ab743ceu));
    p = std::fmaf(r, p, bitsf(0x3c088908u));
    p = std::fmaf(r, p, bitsf(0x3d2aa9c1u));
    p = std::fmaf(r, p, bitsf(0x3e2aaaaau));
    p = std::fmaf(r, p, 0.5f);
    float y = std::fmaf(r * r, p, r);
    float s = bitsf((uint32_t)(((int32_t)k << 23) + 0x3f800000));
    return std::fmaf(s, y, s);
}

#if defined(__AVX2__)
// nexp on eight values, each step the same single rounding as above: the
// clamp (max, then min; a NaN takes the lower bound as fmax gives it),
// round to nearest even, the fma chain, the exponent bits from k.
static inline __m256 nexp8(__m256 x) {
    x = _mm256_min_ps(_mm256_max_ps(x, _mm256_set1_ps(bitsf(0xc2b0c0a5u))), _mm256_set1_ps(bitsf(0x42b0c0a5u)));
    const __m256 k = _mm256_round_ps(_mm256_mul_ps(x, _mm256_set1_ps(bitsf(0x3fb8aa3bu))), _MM_FROUND_TO_NEAREST_INT | _MM_FROUND_NO_EXC);
    __m256 r = _mm256_fmadd_ps(k, _mm256_set1_ps(bitsf(0xbf318000u)), x);
    r = _mm256_fmadd_ps(k, _mm256_set1_ps(bitsf(0x395e8083u)), r);
    __m256 p = _mm256_fmadd_ps(_mm256_set1_ps(bitsf(0x39506967u)), r, _mm256_set1_ps(bitsf(0x3ab743ceu)));
    p = _mm256_fmadd_ps(r, p, _mm256_set1_ps(bitsf(0x3c088908u)));
    p = _mm256_fmadd_ps(r, p, _mm256_set1_ps(bitsf(0x3d2aa9c1u)));
    p = _mm256_fmadd_ps(r, p, _mm256_set1_ps(bitsf(0x3e2aaaaau)));
    p = _mm256_fmadd_ps(r, p, _mm256_set1_ps(0.5f));
    const __m256 y = _mm256_fmadd_ps(_mm256_mul_ps(r, r), p, r);
    const __m256 s = _mm256_castsi256_ps(
        _mm256_add_epi32(_mm256_slli_epi32(_mm256_cvttps_epi32(k), 23), _mm256_set1_epi32(0x3f800000)));
    return _mm256_fmadd_ps(s, y, s);
}
#endif

// x[i] / (nexp(-x[i]) + 1) over n values in place (SiLU; the attention
// gate's divide with g = x), each value's ops as the scalar form's.
static void silu_div(float* x, const float* g, int64_t n) {
    int64_t head = 0;  // values done eight at a time
#if defined(__AVX2__)
    head = n / 8 * 8;
    const __m256 one = _mm256_set1_ps(1.0f), neg = _mm256_set1_ps(-0.0f);
    for (int64_t i = 0; i < head; i += 8) {
        const __m256 gv = _mm256_xor_ps(_mm256_loadu_ps(g + i), neg);
        _mm256_storeu_ps(x + i, _mm256_div_ps(_mm256_loadu_ps(x + i), _mm256_add_ps(nexp8(gv), one)));
    }
#endif
    for (int64_t i = head; i < n; i++) x[i] /= nexp(-g[i]) + 1.0f;
}

// crates/needle-engine/src/infer.rs:372-417 (scalar arm 405-416)
float dot16(const float* x, const float* y, int n) {
    float a[4][4] = {{0}};
    for (int c = 0; c < n / 16; c++)
        for (int j = 0; j < 4; j++)
            for (int l = 0; l < 4; l++) {
                int i = c * 16 + j * 4 + l;
                a[j][l] = std::fmaf(x[i], y[i], a[j][l]);
            }
    float t[4];
    for (int l = 0; l < 4; l++) t[l] = ((a[2][l] + a[3][l]) + a[1][l]) + a[0][l];
    return (t[0] + t[1]) + (t[2] + t[3]);
}

// infer.rs:421-423
static inline float rinv(float ss, int n) { return 1.0f / std::sqrt(ss / (float)n + 1e-6f); }

// infer.rs:426-443 (scalar arm); s given as f32 (f16-exact archive values)
void zcn(const float* x, const float* s, float* out, int n) {
    float r = rinv(dot16(x, x, n), n);
    for (int i = 0; i < n; i++) {
        float t = x[i] * r;
        out[i] = std::fmaf(t, s[i], t);
    }
}

// qlinear.rs:77-88, 113-140 (scalar arms): absmax int8, round half away, saturate.
#if defined(__AVX2__)
// Rust's f32::round (half away from zero) on eight values, exactly: the
// truncation (signed zeros kept), or one further from zero when the
// remainder (exact for every finite value) is at least one half;
// infinities pass through.
static inline __m256 round_away8(__m256 v) {
    const __m256 t = _mm256_round_ps(v, _MM_FROUND_TO_ZERO | _MM_FROUND_NO_EXC);
    const __m256 absmask = _mm256_castsi256_ps(_mm256_set1_epi32(0x7fffffff));
    const __m256 f = _mm256_and_ps(_mm256_sub_ps(v, t), absmask);
    const __m256 one = _mm256_or_ps(_mm256_set1_ps(1.0f), _mm256_andnot_ps(absmask, v));  // ±1 with v's sign
    return _mm256_blendv_ps(t, _mm256_add_ps(t, one), _mm256_cmp_ps(f, _mm256_set1_ps(0.5f), _CMP_GE_OQ));
}
#endif

float quant_i8_scalar(const float* x, int n, int8_t* q);

// qlinear.rs:77-88: as quant_i8_scalar; eight values at a time where the
// build has AVX2 and the row holds no NaN (the scalar loop takes those).
float quant_i8(const float* x, int n, int8_t* q) {
#if defined(__AVX2__)
    const __m256 absmask = _mm256_castsi256_ps(_mm256_set1_epi32(0x7fffffff));
    __m256 mv = _mm256_setzero_ps(), nan = _mm256_setzero_ps();
    int i = 0;
    for (; i + 8 <= n; i += 8) {
        const __m256 v = _mm256_loadu_ps(x + i);
        nan = _mm256_or_ps(nan, _mm256_cmp_ps(v, v, _CMP_UNORD_Q));
        mv = _mm256_max_ps(mv, _mm256_and_ps(v, absmask));
    }
    bool any_nan = _mm256_movemask_ps(nan) != 0;
    alignas(32) float mm[8];
    _mm256_store_ps(mm, mv);
    float m = 0.f;
    for (int k = 0; k < 8; k++) m = rmax(m, mm[k]);  // max is exact in any order
    for (; i < n; i++) {
        any_nan |= x[i] != x[i];
        m = rmax(m, std::fabs(x[i]));
    }
    if (any_nan) return quant_i8_scalar(x, n, q);
    const float s = m > 0.f ? m * K127 : 1.0f;
    const float inv = 1.0f / s;
    const __m256 iv = _mm256_set1_ps(inv), lo = _mm256_set1_ps(-128.f), hi = _mm256_set1_ps(127.f);
    i = 0;
    for (; i + 8 <= n; i += 8) {
        // a NaN product (an infinite element times a zero inverse) gives 0,
        // as the scalar loop's saturating conversion does
        const __m256 p = _mm256_mul_ps(_mm256_loadu_ps(x + i), iv);
        const __m256 r = _mm256_andnot_ps(_mm256_cmp_ps(p, p, _CMP_UNORD_Q),
                                          _mm256_min_ps(_mm256_max_ps(round_away8(p), lo), hi));
        const __m256i w = _mm256_cvttps_epi32(r);
        const __m256i b = _mm256_packs_epi16(_mm256_packs_epi32(w, w), _mm256_setzero_si256());  // bytes 0-3 | 16-19
        const int32_t lo4 = _mm_cvtsi128_si32(_mm256_castsi256_si128(b)), hi4 = _mm_cvtsi128_si32(_mm256_extracti128_si256(b, 1));
        std::memcpy(q + i, &lo4, 4);
        std::memcpy(q + i + 4, &hi4, 4);
    }
    for (; i < n; i++) {
        float v = rround(x[i] * inv);
        v = std::min(std::max(v, -128.f), 127.f);
        q[i] = v != v ? 0 : (int8_t)v;
    }
    return s;
#else
    return quant_i8_scalar(x, n, q);
#endif
}

// qlinear.rs:77-88
float quant_i8_scalar(const float* x, int n, int8_t* q) {
    float m = 0.f;
    for (int i = 0; i < n; i++) m = rmax(m, std::fabs(x[i]));
    float s = m > 0.f ? m * K127 : 1.0f;
    float inv = 1.0f / s;
    for (int i = 0; i < n; i++) {
        float v = rround(x[i] * inv);
        v = std::min(std::max(v, -128.f), 127.f);
        q[i] = v != v ? 0 : (int8_t)v;  // NaN: Rust's saturating `as i8` gives 0
    }
    return s;
}

// ------------------------------------------------------------ quant.rs

// crates/needle-core/src/quant.rs:19-47 — the reference's Lloyd-Max
// centroids as exact f64 bit patterns (a data table that must match).
static const uint64_t LM2[4] = {0xbff81b52e4028034ull, 0xbfdce467275b97c2ull, 0x3fdcfd177c54d348ull, 0x3ff828af1c856640ull};
static const uint64_t LM3[8] = {0xc00121468f3c6b81ull, 0xbff556e7125deacaull, 0xbfe7f2e0f9d592abull, 0xbfce6e4509e1aa2cull,
                                0x3fd000bb25e4dfa5ull, 0x3fe82dc469b936a5ull, 0x3ff568607ac227c5ull, 0x40012e5beccc8fdaull};
static const uint64_t LM4[16] = {0xc005ae0f408928fbull, 0xc0005b0b8a516d54ull, 0xbff9841ff0758fc8ull, 0xbff3bbbebadac679ull,
                                 0xbfed82c6dd21f59eull, 0xbfe47717151708b5ull, 0xbfd7d9b9e4b565faull, 0xbfbd4ca474b8559bull,
                                 0x3fc2683e9154fce2ull, 0x3fd9daf49368793aull, 0x3fe586b43e57d29dull, 0x3feec3d50cbc3b33ull,
                                 0x3ff4688db93b85f1ull, 0x3ffa3164906b428full, 0x4000ace7bbde2442ull, 0x4005ed98d06f2a4aull};

static double d_of(uint64_t b) { double d; std::memcpy(&d, &b, 8); return d; }

// quant.rs:50-68
std::vector<float> codebook(int bits, int group) {
    std::vector<double> c;
    if (bits == 2) for (auto b : LM2) c.push_back(d_of(b));
    else if (bits == 3) for (auto b : LM3) c.push_back(d_of(b));
    else if (bits == 4) for (auto b : LM4) c.push_back(d_of(b));
    else if (bits == 5) c = {-1.2240064, 0.0, 1.2240064};
    else throw std::runtime_error("no CQ codebook");
    double s = std::sqrt((double)group);
    std::vector<float> out;
    for (double v : c) out.push_back((float)(v / s));
    return out;
}

// quant.rs:71-73
static inline float hadamard_scale(int n) { return (float)(1.0 / std::sqrt((double)n)); }

void fwht_scalar(float* x, int n);

// quant.rs:91-105: as fwht_scalar; a 128-point transform eight values at a
// time where the build has AVX2 (a stage's butterflies are independent, and
// each output is the same single add or subtract of the same two values).
void fwht(float* x, int n) {
#if defined(__AVX2__)
    if (n == 128) {
        __m256 v[16];
        for (int k = 0; k < 16; k++) v[k] = _mm256_loadu_ps(x + 8 * k);
        // h = 1, 2, 4 inside a vector: s holds each element's partner; the
        // lower element takes x + s (= a + b), the upper s - x (= a - b)
        const __m256 up1 = _mm256_castsi256_ps(_mm256_setr_epi32(0, -1, 0, -1, 0, -1, 0, -1));
        const __m256 up2 = _mm256_castsi256_ps(_mm256_setr_epi32(0, 0, -1, -1, 0, 0, -1, -1));
        const __m256 up4 = _mm256_castsi256_ps(_mm256_setr_epi32(0, 0, 0, 0, -1, -1, -1, -1));
        for (int k = 0; k < 16; k++) {
            __m256 t = v[k], sw = _mm256_permute_ps(t, 0xB1);
            t = _mm256_blendv_ps(_mm256_add_ps(t, sw), _mm256_sub_ps(sw, t), up1);
            sw = _mm256_permute_ps(t, 0x4E);
            t = _mm256_blendv_ps(_mm256_add_ps(t, sw), _mm256_sub_ps(sw, t), up2);
            sw = _mm256_permute2f128_ps(t, t, 1);
            v[k] = _mm256_blendv_ps(_mm256_add_ps(t, sw), _mm256_sub_ps(sw, t), up4);
        }
        for (int hv = 1; hv < 16; hv *= 2)  // h = 8 hv: whole vectors
            for (int i = 0; i < 16; i += 2 * hv)
                for (int j = i; j < i + hv; j++) {
                    const __m256 a = v[j], b = v[j + hv];
                    v[j] = _mm256_add_ps(a, b);
                    v[j + hv] = _mm256_sub_ps(a, b);
                }
        for (int k = 0; k < 16; k++) _mm256_storeu_ps(x + 8 * k, v[k]);
        return;
    }
#endif
    fwht_scalar(x, n);
}

void fwht_scalar(float* x, int n) {
    for (int h = 1; h < n; h *= 2)
        for (int i = 0; i < n; i += 2 * h)
            for (int j = i; j < i + h; j++) {
                float a = x[j], b = x[j + h];
                x[j] = a + b;
                x[j + h] = a - b;
            }
}

// quant.rs:109-115
void rotate(float* x, int n) {
    fwht(x, n);
    float s = hadamard_scale(n);
    for (int i = 0; i < n; i++) x[i] *= s;
}

// quant.rs:119-124
int nearest(float x, const float* cb, int n) {
    int pos = 0;
    while (pos < n && cb[pos] < x) pos++;
    pos = std::min(std::max(pos, 1), n - 1);
    float l = cb[pos - 1], r = cb[pos];
    return std::fabs(x - l) <= std::fabs(x - r) ? pos - 1 : pos;
}

// quant.rs:127-135
static float quantize_group(float* g, const float* cb, int ncb, uint8_t* idx) {
    rotate(g, GROUP);
    float ss = 0.f;
    for (int i = 0; i < GROUP; i++) ss = ss + g[i] * g[i];
    float norm = std::sqrt(ss);
    float denom = rmax(norm, 1e-12f);
    for (int i = 0; i < GROUP; i++) idx[i] = (uint8_t)nearest(g[i] / denom, cb, ncb);
    return norm;
}

// quant.rs:185-198 (4-bit: byte j = idx[2j] | idx[2j+1] << 4)
static void pack_lsb4(const uint8_t* idx, int n, uint8_t* out) {
    for (int j = 0; j < n / 2; j++) out[j] = (uint8_t)(idx[2 * j] | (idx[2 * j + 1] << 4));
}

// quant.rs:233-256 (bits = 4)
void cq_pack(const float* w, int rows, int d, uint8_t* packed, uint16_t* norms) {
    std::vector<float> cb = codebook(4, GROUP);
    int in_pad = (d + GROUP - 1) / GROUP * GROUP, groups = in_pad / GROUP;
    int per_row = in_pad / 2;
    std::vector<uint8_t> idx(in_pad);
    float g[GROUP];
    for (int r = 0; r < rows; r++) {
        const float* src = w + (size_t)r * d;
        for (int gi = 0; gi < groups; gi++) {
            int start = gi * GROUP, take = std::min(GROUP, std::max(0, d - start));
            for (int i = 0; i < GROUP; i++) g[i] = i < take ? src[start + i] : 0.f;
            float norm = quantize_group(g, cb.data(), (int)cb.size(), idx.data() + start);
            norms[(size_t)r * groups + gi] = f32_to_f16(norm);
        }
        pack_lsb4(idx.data(), in_pad, packed + (size_t)r * per_row);
    }
}

// --------------------------------------------------------------- rng.rs

// crates/needle-core/src/rng.rs:4-74
struct Mt19937 {
    uint32_t mt[624];
    int idx;
    explicit Mt19937(uint32_t seed) {
        mt[0] = seed;
        for (int i = 1; i < 624; i++) mt[i] = 1812433253u * (mt[i - 1] ^ (mt[i - 1] >> 30)) + (uint32_t)i;
        idx = 624;
    }
    void twist() {
        for (int i = 0; i < 624; i++) {
            uint32_t y = (mt[i] & 0x80000000u) | (mt[(i + 1) % 624] & 0x7fffffffu);
            uint32_t v = mt[(i + 397) % 624] ^ (y >> 1);
            if (y & 1) v ^= 0x9908b0dfu;
            mt[i] = v;
        }
        idx = 0;
    }
    uint32_t next() {
        if (idx >= 624) twist();
        uint32_t y = mt[idx++];
        y ^= y >> 11;
        y ^= (y << 7) & 0x9d2c5680u;
        y ^= (y << 15) & 0xefc60000u;
        return y ^ (y >> 18);
    }
    uint32_t interval(uint32_t max) {
        if (max == 0) return 0;
        uint32_t mask = max;
        mask |= mask >> 1; mask |= mask >> 2; mask |= mask >> 4; mask |= mask >> 8; mask |= mask >> 16;
        for (;;) {
            uint32_t v = next() & mask;
            if (v <= max) return v;
        }
    }
    std::vector<int64_t> permutation(int n) {
        std::vector<int64_t> a(n);
        for (int i = 0; i < n; i++) a[i] = i;
        for (int i = n - 1; i >= 1; i--) std::swap(a[i], a[interval((uint32_t)i)]);
        return a;
    }
};

// ------------------------------------------------------------ cact.rs

// crates/needle-core/src/cact.rs:18-22, 47-244
static const uint32_t TAG = 0x05E12A84u;
static const uint32_t TAG_V2 = 0x05E12A83u;
static const int HEADER_BYTES = 49 * 4;
static const int REC_SIZE = 44;
enum Dtype { F16 = 1, F32 = 2, CQ = 3, RAW = 4 };

struct Record {
    int dtype;
    std::vector<int64_t> shape;
    uint64_t offset, nbytes;
    uint32_t group, bits;
};

struct Header {
    uint32_t u[49];
    uint32_t num_tensors() const { return u[1]; }
};

struct Archive {
    const uint8_t* data;
    size_t len;
    uint32_t h[49];
    std::vector<float> cb;
    std::vector<Record> recs;
    const uint8_t* bytes(size_t i) const { return data + recs[i].offset; }
};

static uint32_t rd32(const uint8_t* p) { uint32_t v; std::memcpy(&v, p, 4); return v; }
static uint64_t rd64(const uint8_t* p) { uint64_t v; std::memcpy(&v, p, 8); return v; }

// cact.rs:122-165 (Header::parse), 230-243 (Record::parse), 580-601 (Archive::parse)
void parse_archive(const uint8_t* data, size_t len, Archive& a) {
    if (len < (size_t)HEADER_BYTES) throw std::runtime_error("not a complete .cact archive");
    uint32_t tag = rd32(data);
    if (tag != TAG) {
        if (tag == TAG_V2) throw std::runtime_error("this is a Needle 2 archive; Needle 3 is required");
        throw std::runtime_error("unknown .cact format tag");
    }
    for (int i = 0; i < 49; i++) a.h[i] = rd32(data + 4 * i);
    if (a.h[26] > 4 || a.h[31] > 16) throw std::runtime_error("corrupt .cact header");
    a.data = data;
    a.len = len;
    size_t off = HEADER_BYTES;
    size_t cbn = a.h[2];
    if (off + cbn * 4 > len) throw std::runtime_error("truncated codebook");
    a.cb.resize(cbn);
    for (size_t i = 0; i < cbn; i++) a.cb[i] = bitsf(rd32(data + off + 4 * i));
    off += cbn * 4;
    a.recs.clear();
    for (uint32_t i = 0; i < a.h[1]; i++) {
        if (off + REC_SIZE > len) throw std::runtime_error("truncated directory");
        const uint8_t* b = data + off;
        Record r;
        int nd = b[1];
        if (nd > 4) throw std::runtime_error("corrupt .cact record");
        r.dtype = b[0];
        if (r.dtype < 1 || r.dtype > 4) throw std::runtime_error("unknown .cact tensor dtype");
        for (int k = 0; k < nd; k++) r.shape.push_back(rd32(b + 4 + 4 * k));
        r.offset = rd64(b + 20);
        r.nbytes = rd64(b + 28);
        r.group = rd32(b + 36);
        r.bits = rd32(b + 40);
        if (r.offset + r.nbytes > len) throw std::runtime_error("tensor past the end of the archive");
        a.recs.push_back(r);
        off += REC_SIZE;
    }
}

// ---------------------------------------------------------- qlinear.rs

// quant.rs:11-12: record bits that mark ternary codes (2-bit crumbs).
static const int TERNARY = 5;

// qlinear.rs:222-224: bits a code takes in memory.
static int code_width(int bits) {
    if (bits == TERNARY) return 2;
    if (bits >= 2 && bits <= 4) return bits;
    throw std::runtime_error("CQ records of this width are not supported");
}

// quant.rs:208-225 (unpack_lsb_into): n codes of `width` bits, LSB-first,
// 8 codes per `width` bytes.
static void unpack_lsb(const uint8_t* packed, int width, int n, uint8_t* out) {
    for (int k = 0; k < n; k += 8) {
        uint64_t word = 0;
        for (int b = 0; b < width; b++) word |= (uint64_t)packed[k / 8 * width + b] << (8 * b);
        for (int i = 0; i < 8 && k + i < n; i++) out[k + i] = (uint8_t)((word >> (i * width)) & ((1u << width) - 1));
    }
}

// qlinear.rs:43-61, 211-265, 500-518: a CQ matrix, codes kept as stored,
// plus its codebook. A fused projection concatenates parts of one code
// width; each part keeps its own codebook (QLinear's parts), looked up by
// output row.
struct QPart {
    int r0 = 0;
    int8_t vals[16];
    uint8_t vals_b[16];  // vals + 128, as unsigned bytes
    float cbs;
    float fvals[16];
};

struct QMat {
    int out = 0, in_dim = 0, groups = 0;
    int width = 4;               // bits per code in memory
    std::vector<uint8_t> codes;  // [out][groups][16 * width]
    std::vector<uint16_t> norms; // [out][groups] f16 bits
    std::vector<float> normf;    // the same norms widened (exact)
    std::vector<int8_t> w8;      // codes expanded through `vals`, natural order
    std::vector<QPart> parts;
    bool no_min = false;         // no part's `vals` holds -128
    const QPart& part(int r) const {
        size_t k = parts.size() - 1;
        while (k > 0 && parts[k].r0 > r) k--;
        return parts[k];
    }
};

// qlinear.rs:211-216
static void int8_codebook(const std::vector<float>& cb, int8_t* out, float* scale) {
    float m = 0.f;
    for (float v : cb) m = rmax(m, std::fabs(v));
    float s = m > 0.f ? m * K127 : 1.0f;
    float inv = 1.0f / s;
    for (size_t i = 0; i < cb.size(); i++) {
        float v = std::min(std::max(rround(cb[i] * inv), -128.f), 127.f);
        out[i] = (int8_t)v;
    }
    *scale = s;
}

// qlinear.rs:220-236, 244-265: the codebook of record bits `bits`
// (ternary codes 3, 0, 1 select its centroids 0, 1, 2; a code past the
// codebook reads 0), then codes and norms as stored.
static void qmat_init(QMat& q, int bits, int out, int in_dim, const uint8_t* codes, const uint16_t* norms) {
    q.width = code_width(bits);
    q.out = out;
    q.in_dim = in_dim;
    q.groups = (in_dim + GROUP - 1) / GROUP;
    const size_t bpg = 16 * (size_t)q.width, ncode = (size_t)out * q.groups * bpg;
    q.codes.assign(codes, codes + ncode);
    q.norms.assign(norms, norms + (size_t)out * q.groups);
    q.normf.resize(q.norms.size());
    for (size_t i = 0; i < q.norms.size(); i++) q.normf[i] = f16_to_f32(q.norms[i]);
    std::vector<float> cb = codebook(bits, GROUP);
    int8_t cb8[16];
    QPart pt;
    int8_codebook(cb, cb8, &pt.cbs);
    for (int c = 0; c < 16; c++) {
        int k = bits == TERNARY ? (c == 3 ? 0 : c + 1) : c;
        bool in = c < (1 << q.width) && k < (int)cb.size();
        pt.vals[c] = in ? cb8[k] : 0;
        pt.vals_b[c] = (uint8_t)(pt.vals[c] + 128);
        pt.fvals[c] = in ? cb[k] : 0.f;
    }
    q.parts.assign(1, pt);
    q.no_min = true;
    for (int c = 0; c < 16; c++) q.no_min &= pt.vals[c] != -128;
    q.w8.resize((size_t)out * q.groups * GROUP);
    uint8_t idx[GROUP];
    for (size_t u = 0; u < (size_t)out * q.groups; u++) {
        unpack_lsb(q.codes.data() + u * bpg, q.width, GROUP, idx);
        for (int p = 0; p < GROUP; p++) q.w8[u * GROUP + p] = pt.vals[idx[p]];
    }
}

static void qmat_from_cq(const Archive& a, size_t i, QMat& q) {
    const Record& r = a.recs[i];
    if (r.dtype != CQ) throw std::runtime_error("tensor is not CQ");
    if (r.group != (uint32_t)GROUP) throw std::runtime_error("CQ group size is not supported");
    int out = (int)r.shape[0], in_dim = (int)r.shape[1], groups = (in_dim + GROUP - 1) / GROUP;
    size_t ncode = (size_t)out * groups * 16 * code_width((int)r.bits);
    if (r.nbytes < ncode + (size_t)out * groups * 2) throw std::runtime_error("CQ record is truncated");
    const uint8_t* blob = a.bytes(i);
    std::vector<uint16_t> nr((size_t)out * groups);
    std::memcpy(nr.data(), blob + ncode, nr.size() * 2);
    qmat_init(q, (int)r.bits, out, in_dim, blob, nr.data());
}

// qlinear.rs:503-518: parts side by side; the code width must agree.
static void qmat_concat(QMat& dst, const QMat& src) {
    if (dst.out == 0) { dst = src; return; }
    if (dst.width != src.width) throw std::runtime_error("fused parts must share a code width");
    for (QPart p : src.parts) {
        p.r0 += dst.out;
        dst.parts.push_back(p);
    }
    dst.out += src.out;
    dst.no_min = dst.no_min && src.no_min;
    dst.codes.insert(dst.codes.end(), src.codes.begin(), src.codes.end());
    dst.norms.insert(dst.norms.end(), src.norms.begin(), src.norms.end());
    dst.normf.insert(dst.normf.end(), src.normf.begin(), src.normf.end());
    dst.w8.insert(dst.w8.end(), src.w8.begin(), src.w8.end());
}

// qlinear.rs:309-323
static void qmat_row(const QMat& q, int r, float* out) {
    std::vector<float> buf((size_t)q.groups * GROUP);
    const QPart& pt = q.part(r);
    uint8_t idx[GROUP];
    for (int g = 0; g < q.groups; g++) {
        float norm = f16_to_f32(q.norms[(size_t)r * q.groups + g]);
        float* dst = buf.data() + g * GROUP;
        unpack_lsb(q.codes.data() + ((size_t)r * q.groups + g) * 16 * q.width, q.width, GROUP, idx);
        for (int p = 0; p < GROUP; p++) dst[p] = pt.fvals[idx[p]] * norm;
        rotate(dst, GROUP);
    }
    std::memcpy(out, buf.data(), sizeof(float) * q.in_dim);
}

// qlinear.rs:65-72: activations, stored here in natural order (the
// reference's de-interleaved layout only permutes exact integer sums).
struct QAct {
    int rows = 0, groups = 0;
    std::vector<int8_t> xq;  // [rows][groups*128], natural order
    std::vector<float> sx;   // [rows][groups]
    // xq widened to int16, each 32-wide block as its 16 even elements then
    // its 16 odd ones (the order the 4-bit code bytes hold the weights in)
    std::vector<int16_t> xeo;
    // xq as int8 and as magnitudes, each pair of 32-wide blocks as the even
    // elements of both, then the odd elements of both; no_min: xq holds no
    // -128 (every magnitude fits a signed byte)
    std::vector<int8_t> x8eo;
    std::vector<uint8_t> ax8eo;
    bool no_min = false;
    // each group's 64 even elements, then its 64 odd ones; and per group the
    // sums of xq over the four 4-bit decode lanes (lane (p % 32) / 8)
    std::vector<int8_t> x8v;
    std::vector<int32_t> sumx;  // [rows][groups][4]
};

// qlinear.rs:152-164
float prep_group(const float* x, int n, int g, int8_t* q) {
    float buf[GROUP];
    int start = g * GROUP, take = std::min(GROUP, n - start);
    for (int i = 0; i < GROUP; i++) buf[i] = i < take ? x[start + i] : 0.f;
    rotate(buf, GROUP);
    return quant_i8(buf, GROUP, q);
}

// qlinear.rs:191-207
static QAct qact_new(const float* x, int rows, int in_dim) {
    QAct a;
    a.rows = rows;
    a.groups = (in_dim + GROUP - 1) / GROUP;
    a.xq.assign((size_t)rows * a.groups * GROUP, 0);
    a.sx.assign((size_t)rows * a.groups, 0.f);
    for (int r = 0; r < rows; r++)
        for (int g = 0; g < a.groups; g++)
            a.sx[(size_t)r * a.groups + g] =
                prep_group(x + (size_t)r * in_dim, in_dim, g, a.xq.data() + ((size_t)r * a.groups + g) * GROUP);
    // the layouts the host's 4-bit path reads: VNNI's, or AVX2's
    if (vnni_host()) {
        a.x8v.resize(a.xq.size());
        a.sumx.assign(a.xq.size() / GROUP * 4, 0);
        for (size_t g = 0; g < a.xq.size() / GROUP; g++)
            for (int p = 0; p < GROUP; p++) {
                const int8_t v = a.xq[g * GROUP + p];
                a.x8v[g * GROUP + (p & 1) * 64 + p / 2] = v;
                a.sumx[g * 4 + (p % 32) / 8] += v;
            }
        return a;
    }
    a.xeo.resize(a.xq.size());
    for (size_t b = 0; b < a.xq.size(); b += 32)
        for (int j = 0; j < 16; j++) {
            a.xeo[b + j] = a.xq[b + 2 * j];
            a.xeo[b + 16 + j] = a.xq[b + 2 * j + 1];
        }
    a.x8eo.resize(a.xq.size());
    a.ax8eo.resize(a.xq.size());
    a.no_min = true;
    for (size_t b = 0; b < a.xq.size(); b += 64)  // two 32-wide blocks
        for (int h = 0; h < 2; h++)
            for (int j = 0; j < 16; j++)
                for (int odd = 0; odd < 2; odd++) {
                    const int8_t v = a.xq[b + 32 * h + 2 * j + odd];
                    const size_t at = b + 32 * odd + 16 * h + j;
                    a.x8eo[at] = v;
                    a.ax8eo[at] = (uint8_t)std::abs((int)v);
                    a.no_min &= v != -128;
                }
    return a;
}

// qlinear.rs:327-337: the 4 decode lanes of one group of 128 int8 weights
// w and activations x (natural order); lane = (p % 64) / 16 for 2-bit
// codes, (p % 32) / 8 otherwise.
static inline void lane_sums_scalar(const int8_t* w, const int8_t* x, int width, int32_t s[4]) {
    if (width == 2) {  // lane l: p = 64h + 16l + b
        for (int l = 0; l < 4; l++) {
            int32_t acc = 0;
            for (int h = 0; h < 2; h++) {
                const int8_t* wp = w + h * 64 + l * 16;
                const int8_t* xp = x + h * 64 + l * 16;
                for (int b = 0; b < 16; b++) acc += (int32_t)wp[b] * (int32_t)xp[b];
            }
            s[l] = acc;
        }
        return;
    }
    for (int l = 0; l < 4; l++) {  // lane l: p = 32a + 8l + b
        int32_t acc = 0;
        for (int blk = 0; blk < 4; blk++) {
            const int8_t* wp = w + blk * 32 + l * 8;
            const int8_t* xp = x + blk * 32 + l * 8;
            for (int b = 0; b < 8; b++) acc += (int32_t)wp[b] * (int32_t)xp[b];
        }
        s[l] = acc;
    }
}

#if defined(__AVX2__)
static inline int32_t hsum_i32x4(__m128i v) {
    v = _mm_add_epi32(v, _mm_shuffle_epi32(v, 0x4E));
    v = _mm_add_epi32(v, _mm_shuffle_epi32(v, 0xB1));
    return _mm_cvtsi128_si32(v);
}

// lane_sums_scalar's integer sums, sixteen products at a time: int8 widened
// to int16, adjacent products summed into int32 (vpmaddwd, exact: no
// saturation), a lane's pair sums added at the end. Integer addition is
// exact in any order, so the sums are the scalar ones.
static inline void lane_sums_avx2(const int8_t* w, const int8_t* x, int width, int32_t s[4]) {
    auto prod16 = [](const int8_t* a, const int8_t* b) {
        __m256i a16 = _mm256_cvtepi8_epi16(_mm_loadu_si128((const __m128i*)a));
        __m256i b16 = _mm256_cvtepi8_epi16(_mm_loadu_si128((const __m128i*)b));
        return _mm256_madd_epi16(a16, b16);  // int32 i: products 2i and 2i + 1
    };
    if (width == 2) {  // lane l: bytes 64h + 16l .. + 15
        for (int l = 0; l < 4; l++) {
            __m256i acc = _mm256_add_epi32(prod16(w + l * 16, x + l * 16), prod16(w + 64 + l * 16, x + 64 + l * 16));
            s[l] = hsum_i32x4(_mm_add_epi32(_mm256_castsi256_si128(acc), _mm256_extracti128_si256(acc, 1)));
        }
        return;
    }
    // lane l: bytes 32a + 8l .. + 7; a 16-byte half of a 32-byte block
    // holds two lanes, one in each 128-bit half of the int32 pair sums
    __m256i a01 = _mm256_setzero_si256(), a23 = _mm256_setzero_si256();
    for (int blk = 0; blk < 4; blk++) {
        a01 = _mm256_add_epi32(a01, prod16(w + blk * 32, x + blk * 32));
        a23 = _mm256_add_epi32(a23, prod16(w + blk * 32 + 16, x + blk * 32 + 16));
    }
    s[0] = hsum_i32x4(_mm256_castsi256_si128(a01));
    s[1] = hsum_i32x4(_mm256_extracti128_si256(a01, 1));
    s[2] = hsum_i32x4(_mm256_castsi256_si128(a23));
    s[3] = hsum_i32x4(_mm256_extracti128_si256(a23, 1));
}
#endif

// Σ a[e] b[e] over n int8 pairs, exact (int32; any order).
static inline int32_t dot_i8(const int8_t* a, const int8_t* b, int n) {
    int e = 0;
    int32_t acc = 0;
#if defined(__AVX2__)
    __m256i v = _mm256_setzero_si256();
    for (; e + 16 <= n; e += 16)
        v = _mm256_add_epi32(v, _mm256_madd_epi16(_mm256_cvtepi8_epi16(_mm_loadu_si128((const __m128i*)(a + e))),
                                                  _mm256_cvtepi8_epi16(_mm_loadu_si128((const __m128i*)(b + e)))));
    acc = hsum_i32x4(_mm_add_epi32(_mm256_castsi256_si128(v), _mm256_extracti128_si256(v, 1)));
#endif
    for (; e < n; e++) acc += (int32_t)a[e] * (int32_t)b[e];
    return acc;
}

static inline void lane_sums_of(const int8_t* w, const int8_t* x, int width, int32_t s[4]) {
#if defined(__AVX2__)
    lane_sums_avx2(w, x, width, s);
#else
    lane_sums_scalar(w, x, width, s);
#endif
}

#if defined(__AVX2__)
// The lane sums of a 4-bit group read from its 64 code bytes (byte k holds
// the codes of p = 2k, low nibble, and 2k + 1) against the group's
// activations as QAct::xeo holds them: the codebook's int8 values looked up
// sixteen at a time (pshufb) for the even and for the odd elements of a
// 32-wide block, widened, multiplied with the matching activations and
// summed in pairs into int32 (vpmaddwd, exact); in a block, code bytes
// 4l .. 4l + 3 are lane l's, so int32 pair sums 2l and 2l + 1 are too. The
// same exact integers as expanding the codes through `vals` first.
static inline void lane_sums_codes4_avx2(const uint8_t* codes, const int8_t* vals, const int16_t* xeo, int32_t s[4]) {
    const __m128i tbl = _mm_loadu_si128((const __m128i*)vals), m4 = _mm_set1_epi8(0x0F);
    __m256i acc = _mm256_setzero_si256();
    for (int blk = 0; blk < 4; blk++) {
        const __m128i c = _mm_loadu_si128((const __m128i*)(codes + 16 * blk));
        const __m256i we = _mm256_cvtepi8_epi16(_mm_shuffle_epi8(tbl, _mm_and_si128(c, m4)));
        const __m256i wo = _mm256_cvtepi8_epi16(_mm_shuffle_epi8(tbl, _mm_and_si128(_mm_srli_epi16(c, 4), m4)));
        acc = _mm256_add_epi32(acc, _mm256_madd_epi16(we, _mm256_loadu_si256((const __m256i*)(xeo + 32 * blk))));
        acc = _mm256_add_epi32(acc, _mm256_madd_epi16(wo, _mm256_loadu_si256((const __m256i*)(xeo + 32 * blk + 16))));
    }
    const __m256i h = _mm256_hadd_epi32(acc, acc);  // lanes 0, 1 in the low half, 2, 3 in the high
    alignas(32) int32_t v[8];
    _mm256_store_si256((__m256i*)v, h);
    s[0] = v[0];
    s[1] = v[1];
    s[2] = v[4];
    s[3] = v[5];
}
#endif

#if defined(__AVX2__)
// lane_sums_codes4_avx2's integers two 32-wide blocks at a time, when no
// weight value and no activation is -128: byte products |x| * (w signed by
// x) summed in pairs into int16 (vpmaddubsw: a pair is at most 2 * 127 *
// 127 = 32258, so nothing saturates), then pairs of those into int32. In a
// 128-bit half (one block) int32 m is lane m. x8/ax8: the group's
// activations and magnitudes as QAct::x8eo / ax8eo hold them; tbl: `vals`
// in both 128-bit halves. Returns the four lanes.
static inline __m128i lane_sums_codes4_ub(const uint8_t* codes, __m256i tbl, const int8_t* x8, const uint8_t* ax8) {
    const __m256i m4 = _mm256_set1_epi8(0x0F), ones = _mm256_set1_epi16(1);
    __m256i acc = _mm256_setzero_si256();
    for (int pr = 0; pr < 2; pr++) {
        const __m256i c = _mm256_loadu_si256((const __m256i*)(codes + 32 * pr));
        const __m256i we = _mm256_shuffle_epi8(tbl, _mm256_and_si256(c, m4));
        const __m256i wo = _mm256_shuffle_epi8(tbl, _mm256_and_si256(_mm256_srli_epi16(c, 4), m4));
        const __m256i xe = _mm256_loadu_si256((const __m256i*)(x8 + 64 * pr));
        const __m256i xo = _mm256_loadu_si256((const __m256i*)(x8 + 64 * pr + 32));
        const __m256i pe = _mm256_maddubs_epi16(_mm256_loadu_si256((const __m256i*)(ax8 + 64 * pr)), _mm256_sign_epi8(we, xe));
        const __m256i po = _mm256_maddubs_epi16(_mm256_loadu_si256((const __m256i*)(ax8 + 64 * pr + 32)), _mm256_sign_epi8(wo, xo));
        acc = _mm256_add_epi32(acc, _mm256_add_epi32(_mm256_madd_epi16(pe, ones), _mm256_madd_epi16(po, ones)));
    }
    return _mm_add_epi32(_mm256_castsi256_si128(acc), _mm256_extracti128_si256(acc, 1));
}
#endif

#if defined(__AVX2__) && defined(__x86_64__)
// AVX-512 VNNI, chosen at run time where the host has it (the rest of this
// file needs only AVX2).
#define ORC_VNNI __attribute__((target("avx512f,avx512bw,avx512vl,avx512vnni")))
static const bool g_vnni = vnni_host();

// The four lane sums of a 4-bit group from its 64 code bytes: the codebook
// looked up sixty-four codes at a time into unsigned bytes w + 128 (tblb:
// vals_b in every 128-bit quarter), then vpdpbusd adds each four adjacent
// (w + 128) * x byte products into an int32, exactly (no saturation). In
// the even and the odd half alike int32 e holds p in [8e, 8e + 8), lane
// e % 4, so the four quarters summed are the lanes, less 128 times the
// lane's activation sum. x8v, sumx4: the group as QAct::x8v / sumx hold it.
ORC_VNNI static inline __m128i lane_sums_codes4_vnni(const uint8_t* codes, __m512i tblb, const int8_t* x8v, __m128i sumx4) {
    const __m512i c = _mm512_loadu_si512(codes), m4 = _mm512_set1_epi8(0x0F);
    const __m512i we = _mm512_shuffle_epi8(tblb, _mm512_and_si512(c, m4));
    const __m512i wo = _mm512_shuffle_epi8(tblb, _mm512_and_si512(_mm512_srli_epi16(c, 4), m4));
    __m512i acc = _mm512_dpbusd_epi32(_mm512_setzero_si512(), we, _mm512_loadu_si512(x8v));
    acc = _mm512_dpbusd_epi32(acc, wo, _mm512_loadu_si512(x8v + 64));
    const __m256i h = _mm256_add_epi32(_mm512_castsi512_si256(acc), _mm512_extracti64x4_epi64(acc, 1));
    const __m128i l = _mm_add_epi32(_mm256_castsi256_si128(h), _mm256_extracti128_si256(h, 1));
    return _mm_sub_epi32(l, _mm_slli_epi32(sumx4, 7));
}

ORC_VNNI static void lane_sums_vnni(const uint8_t* codes, const uint8_t* vals_b, const int8_t* x8v, const int32_t* sumx,
                                    int32_t s[4]) {
    _mm_storeu_si128((__m128i*)s, lane_sums_codes4_vnni(codes, _mm512_broadcast_i32x4(_mm_loadu_si128((const __m128i*)vals_b)),
                                                        x8v, _mm_loadu_si128((const __m128i*)sumx)));
}
#else
static const bool g_vnni = false;
#endif

// The lane sums of row r (part pt), group g against activation row t.
static inline void lane_sums(const QMat& q, const QPart& pt, int r, int g, const QAct& a, int t, int32_t s[4]) {
    const size_t ag = ((size_t)t * a.groups + g) * GROUP;
#if defined(__AVX2__) && defined(__x86_64__)
    if (q.width == 4 && g_vnni) {
        lane_sums_vnni(q.codes.data() + ((size_t)r * q.groups + g) * 64, pt.vals_b, a.x8v.data() + ag, a.sumx.data() + ag / GROUP * 4,
                       s);
        return;
    }
#endif
#if defined(__AVX2__)
    if (q.width == 4 && q.no_min && a.no_min) {
        const __m256i tbl = _mm256_broadcastsi128_si256(_mm_loadu_si128((const __m128i*)pt.vals));
        _mm_storeu_si128((__m128i*)s, lane_sums_codes4_ub(q.codes.data() + ((size_t)r * q.groups + g) * 64, tbl,
                                                          a.x8eo.data() + ag, a.ax8eo.data() + ag));
        return;
    }
    if (q.width == 4) {
        lane_sums_codes4_avx2(q.codes.data() + ((size_t)r * q.groups + g) * 64, pt.vals, a.xeo.data() + ag, s);
        return;
    }
#endif
    (void)pt;
    lane_sums_of(q.w8.data() + ((size_t)r * q.groups + g) * GROUP, a.xq.data() + ag, q.width, s);
}

// qlinear.rs:340-350
float decode_row_ref(const QMat& q, int r, const QAct& a) {
    const QPart& pt = q.part(r);
    const float cbs = pt.cbs;
    float lanes[4] = {0.f, 0.f, 0.f, 0.f};
    for (int g = 0; g < q.groups; g++) {
        int32_t s[4];
        lane_sums(q, pt, r, g, a, 0, s);
        float sc = (a.sx[g] * cbs) * q.normf[(size_t)r * q.groups + g];
        for (int l = 0; l < 4; l++) lanes[l] = std::fmaf((float)s[l], sc, lanes[l]);
    }
    return (lanes[0] + lanes[1]) + (lanes[2] + lanes[3]);
}

// qlinear.rs:353-363
float prefill_row_ref(const QMat& q, int r, const QAct& a, int t, bool block) {
    const QPart& pt = q.part(r);
    const float cbs = pt.cbs;
    float acc = 0.f;
    for (int g = 0; g < q.groups; g++) {
        int32_t s[4];
        lane_sums(q, pt, r, g, a, t, s);
        int32_t tot = s[0] + s[1] + s[2] + s[3];
        float sx = a.sx[(size_t)t * a.groups + g];
        float norm = q.normf[(size_t)r * q.groups + g];
        float sc = block ? (norm * cbs) * sx : norm * (cbs * sx);
        acc = std::fmaf((float)tot, sc, acc);
    }
    return acc;
}

// decode_row_ref for every row of q into y[0 .. q.out): with AVX2, eight
// rows side by side, each row's floats the same single ops in the same
// order (its scale product, its four lane fma chains over the groups, the
// final two-level sum).
#if defined(__AVX2__) && defined(__x86_64__)
// decode_rows_range's eight-row blocks of a 4-bit matrix with the lane sums
// on AVX-512 VNNI (lane_sums_codes4_vnni), the floats as there. Returns the
// first row it left (the block tail) for the caller.
ORC_VNNI static int decode_rows_vnni(const QMat& q, const QAct& a, float* y, int r, int r_end) {
    for (; r + 8 <= r_end; r += 8) {
        if (r + 24 <= r_end) {
            const uint8_t* nxt = q.codes.data() + (size_t)(r + 16) * q.groups * 64;
            for (int b = 0; b < 8 * q.groups * 64; b += 64) _mm_prefetch((const char*)(nxt + b), _MM_HINT_T0);
        }
        float cbs[8];
        __m512i tbl[8];
        for (int k = 0; k < 8; k++) {
            const QPart& pt = q.part(r + k);
            cbs[k] = pt.cbs;
            tbl[k] = _mm512_broadcast_i32x4(_mm_loadu_si128((const __m128i*)pt.vals_b));
        }
        const __m256 cbv = _mm256_loadu_ps(cbs);
        __m256 ln[4] = {_mm256_setzero_ps(), _mm256_setzero_ps(), _mm256_setzero_ps(), _mm256_setzero_ps()};
        for (int g = 0; g < q.groups; g++) {
            const size_t ag = (size_t)g * GROUP;
            const __m128i sx4 = _mm_loadu_si128((const __m128i*)(a.sumx.data() + (size_t)g * 4));
            __m128i v[8];  // row k's four lane sums
            for (int k = 0; k < 8; k++)
                v[k] = lane_sums_codes4_vnni(q.codes.data() + ((size_t)(r + k) * q.groups + g) * 64, tbl[k], a.x8v.data() + ag, sx4);
            __m128i lo[4], hi[4];  // transposed: lane l of rows 0..7
            for (int h = 0; h < 2; h++) {
                const __m128i* w = v + 4 * h;
                const __m128i t0 = _mm_unpacklo_epi32(w[0], w[1]), t1 = _mm_unpackhi_epi32(w[0], w[1]);
                const __m128i t2 = _mm_unpacklo_epi32(w[2], w[3]), t3 = _mm_unpackhi_epi32(w[2], w[3]);
                __m128i* o = h ? hi : lo;
                o[0] = _mm_unpacklo_epi64(t0, t2);
                o[1] = _mm_unpackhi_epi64(t0, t2);
                o[2] = _mm_unpacklo_epi64(t1, t3);
                o[3] = _mm_unpackhi_epi64(t1, t3);
            }
            alignas(32) float nf[8];
            for (int k = 0; k < 8; k++) nf[k] = q.normf[(size_t)(r + k) * q.groups + g];
            const __m256 sc = _mm256_mul_ps(_mm256_mul_ps(_mm256_set1_ps(a.sx[g]), cbv), _mm256_load_ps(nf));
            for (int l = 0; l < 4; l++) ln[l] = _mm256_fmadd_ps(_mm256_cvtepi32_ps(_mm256_set_m128i(hi[l], lo[l])), sc, ln[l]);
        }
        _mm256_storeu_ps(y + r, _mm256_add_ps(_mm256_add_ps(ln[0], ln[1]), _mm256_add_ps(ln[2], ln[3])));
    }
    return r;
}
#endif

#if defined(__AVX2__) && defined(__x86_64__)
// prefill_row_ref for rows r .. r_end - 1 (whole eight-row blocks; returns
// the first row left) of a 4-bit matrix and every token t of a, on AVX-512
// VNNI: per token and group the eight rows' lane sums, their totals (exact
// integer adds), the scale by the block or remainder rule and the fma, each
// row's ops as the scalar form's in its order.
ORC_VNNI static int prefill_rows_vnni(const QMat& q, const QAct& a, float* y, int ldy, int col0, int r, int r_end) {
    const int blocked = a.rows / 4 * 4;
    for (; r + 8 <= r_end; r += 8) {
        float cbs[8];
        __m512i tbl[8];
        for (int k = 0; k < 8; k++) {
            const QPart& pt = q.part(r + k);
            cbs[k] = pt.cbs;
            tbl[k] = _mm512_broadcast_i32x4(_mm_loadu_si128((const __m128i*)pt.vals_b));
        }
        const __m256 cbv = _mm256_loadu_ps(cbs);
        for (int t = 0; t < a.rows; t++) {
            __m256 acc = _mm256_setzero_ps();
            for (int g = 0; g < q.groups; g++) {
                const size_t ag = ((size_t)t * a.groups + g) * GROUP;
                const __m128i sx4 = _mm_loadu_si128((const __m128i*)(a.sumx.data() + ag / GROUP * 4));
                __m128i v[8];
                for (int k = 0; k < 8; k++)
                    v[k] = lane_sums_codes4_vnni(q.codes.data() + ((size_t)(r + k) * q.groups + g) * 64, tbl[k], a.x8v.data() + ag, sx4);
                __m128i tot[2];  // rows 0-3, 4-7: the four lanes' sum
                for (int h = 0; h < 2; h++) {
                    const __m128i* w = v + 4 * h;
                    const __m128i t0 = _mm_unpacklo_epi32(w[0], w[1]), t1 = _mm_unpackhi_epi32(w[0], w[1]);
                    const __m128i t2 = _mm_unpacklo_epi32(w[2], w[3]), t3 = _mm_unpackhi_epi32(w[2], w[3]);
                    tot[h] = _mm_add_epi32(_mm_add_epi32(_mm_unpacklo_epi64(t0, t2), _mm_unpackhi_epi64(t0, t2)),
                                           _mm_add_epi32(_mm_unpacklo_epi64(t1, t3), _mm_unpackhi_epi64(t1, t3)));
                }
                alignas(32) float nf[8];
                for (int k = 0; k < 8; k++) nf[k] = q.normf[(size_t)(r + k) * q.groups + g];
                const __m256 nv = _mm256_load_ps(nf), sxv = _mm256_set1_ps(a.sx[(size_t)t * a.groups + g]);
                const __m256 sc = t < blocked ? _mm256_mul_ps(_mm256_mul_ps(nv, cbv), sxv) : _mm256_mul_ps(nv, _mm256_mul_ps(cbv, sxv));
                acc = _mm256_fmadd_ps(_mm256_cvtepi32_ps(_mm256_set_m128i(tot[1], tot[0])), sc, acc);
            }
            _mm256_storeu_ps(y + (size_t)t * ldy + col0 + r, acc);
        }
    }
    return r;
}
#endif

static void decode_rows_range(const QMat& q, const QAct& a, float* y, int r, int r_end) {
#if defined(__AVX2__) && defined(__x86_64__)
    if (q.width == 4 && g_vnni) r = decode_rows_vnni(q, a, y, r, r_end);
#endif
#if defined(__AVX2__)
    for (; r + 8 <= r_end; r += 8) {
        const QPart* pts[8];
        float cbs[8];
        for (int k = 0; k < 8; k++) {
            pts[k] = &q.part(r + k);
            cbs[k] = pts[k]->cbs;
        }
        const __m256 cbv = _mm256_loadu_ps(cbs);
        __m256 ln[4] = {_mm256_setzero_ps(), _mm256_setzero_ps(), _mm256_setzero_ps(), _mm256_setzero_ps()};
        if (q.width == 4 && q.no_min && a.no_min) {
            // the code bytes of the block two blocks on, into the caches
            // while this one is summed (rows r .. r + 7 are contiguous)
            if (r + 24 <= r_end) {
                const uint8_t* nxt = q.codes.data() + (size_t)(r + 16) * q.groups * 64;
                for (int b = 0; b < 8 * q.groups * 64; b += 64) _mm_prefetch((const char*)(nxt + b), _MM_HINT_T0);
            }
            __m256i tbl[8];
            for (int k = 0; k < 8; k++) tbl[k] = _mm256_broadcastsi128_si256(_mm_loadu_si128((const __m128i*)pts[k]->vals));
            for (int g = 0; g < q.groups; g++) {
                const size_t ag = (size_t)g * GROUP;
                __m128i v[8];  // row k's four lane sums
                for (int k = 0; k < 8; k++)
                    v[k] = lane_sums_codes4_ub(q.codes.data() + ((size_t)(r + k) * q.groups + g) * 64, tbl[k], a.x8eo.data() + ag,
                                               a.ax8eo.data() + ag);
                // transposed: lane l of rows 0..7
                __m128i lo[4], hi[4];
                for (int h = 0; h < 2; h++) {
                    const __m128i* w = v + 4 * h;
                    const __m128i t0 = _mm_unpacklo_epi32(w[0], w[1]), t1 = _mm_unpackhi_epi32(w[0], w[1]);
                    const __m128i t2 = _mm_unpacklo_epi32(w[2], w[3]), t3 = _mm_unpackhi_epi32(w[2], w[3]);
                    __m128i* o = h ? hi : lo;
                    o[0] = _mm_unpacklo_epi64(t0, t2);
                    o[1] = _mm_unpackhi_epi64(t0, t2);
                    o[2] = _mm_unpacklo_epi64(t1, t3);
                    o[3] = _mm_unpackhi_epi64(t1, t3);
                }
                alignas(32) float nf[8];
                for (int k = 0; k < 8; k++) nf[k] = q.normf[(size_t)(r + k) * q.groups + g];
                const __m256 sc = _mm256_mul_ps(_mm256_mul_ps(_mm256_set1_ps(a.sx[g]), cbv), _mm256_load_ps(nf));
                for (int l = 0; l < 4; l++)
                    ln[l] = _mm256_fmadd_ps(_mm256_cvtepi32_ps(_mm256_set_m128i(hi[l], lo[l])), sc, ln[l]);
            }
            _mm256_storeu_ps(y + r, _mm256_add_ps(_mm256_add_ps(ln[0], ln[1]), _mm256_add_ps(ln[2], ln[3])));
            continue;
        }
        for (int g = 0; g < q.groups; g++) {
            alignas(32) int32_t s[4][8];
            alignas(32) float nf[8];
            for (int k = 0; k < 8; k++) {
                int32_t t4[4];
                lane_sums(q, *pts[k], r + k, g, a, 0, t4);
                for (int l = 0; l < 4; l++) s[l][k] = t4[l];
                nf[k] = q.normf[(size_t)(r + k) * q.groups + g];
            }
            const __m256 sc = _mm256_mul_ps(_mm256_mul_ps(_mm256_set1_ps(a.sx[g]), cbv), _mm256_load_ps(nf));
            for (int l = 0; l < 4; l++)
                ln[l] = _mm256_fmadd_ps(_mm256_cvtepi32_ps(_mm256_load_si256((const __m256i*)s[l])), sc, ln[l]);
        }
        _mm256_storeu_ps(y + r, _mm256_add_ps(_mm256_add_ps(ln[0], ln[1]), _mm256_add_ps(ln[2], ln[3])));
    }
#endif
    for (; r < r_end; r++) y[r] = decode_row_ref(q, r, a);
}

static void decode_rows(const QMat& q, const QAct& a, float* y) {
    const int blocks = q.out / 8;
    if (q.out < 256) {
        decode_rows_range(q, a, y, 0, q.out);
        return;
    }
    g_team.run(blocks, [&](int b0, int b1) { decode_rows_range(q, a, y, 8 * b0, b1 == blocks ? q.out : 8 * b1); });
}

// qlinear.rs:366-419, 460-487: decode kernel for one token, prefill kernel
// (block tokens t < T/4*4, remainder tokens after) for more.
static void qmat_matmul(const QMat& q, const QAct& a, float* y, int ldy, int col0) {
    if (a.rows == 1) {
        decode_rows(q, a, y + col0);
    } else {
        int blocked = a.rows / 4 * 4;
        const int blocks = (q.out + 7) / 8;
        g_team.run(blocks, [&](int b0, int b1) {
            int r0 = 8 * b0;
            const int r1 = std::min(q.out, 8 * b1);
#if defined(__AVX2__) && defined(__x86_64__)
            if (q.width == 4 && g_vnni) r0 = prefill_rows_vnni(q, a, y, ldy, col0, r0, r1);
#endif
            for (int t = 0; t < a.rows; t++)
                for (int r = r0; r < r1; r++) y[(size_t)t * ldy + col0 + r] = prefill_row_ref(q, r, a, t, t < blocked);
        });
    }
}

// qlinear.rs:454-456
float single_row(const QMat& q, int r, const QAct& a) { return prefill_row_ref(q, r, a, 0, true); }

// ----------------------------------------------------------- the model

struct Config {
    int vocab, out_vocab, d, nh, nkv, L, qk, vd, max_seq, hada_n, lanes, sw;
    uint64_t global_mask;
    int taps, eslots, esub, ntables, etaps, edil, eseed;
    std::vector<int> orders, sites;
    float theta;
    int kv_window, kv_bits;
    int out_rows() const { return out_vocab > 0 ? out_vocab : vocab; }
    int window(int l) const { return (sw > 0 && !((global_mask >> l) & 1)) ? sw : 0; }
    int eheads() const { return orders.empty() ? 0 : ntables / (int)orders.size(); }
};

struct Layer {
    std::vector<float> norm_in, q_taps, k_taps, v_taps, q_norm, k_norm, post_norm, pre_hada;
    float attn_gate;
    std::vector<float> d1, d2, b2, d3, d4, kron[6], cond_v, cond_u;
    float a_pre, a_post, a_res;
    std::vector<float> b_pre, b_post, b_res;
    QMat qkvg, out;
    // infer.rs:852-866: the mHC gate projection, rows requantized to int8.
    int phi_rows, phi_width;
    std::vector<int8_t> phi_q;
    std::vector<float> phi_s;
};

struct Engram {
    QMat tables, kv;
    std::vector<float> taps;
};

struct Model {
    Config c;
    std::vector<uint8_t> bytes;
    QMat embedding;
    std::vector<Layer> layers;
    std::vector<Engram> engrams;
    std::vector<int> site_of_layer;
    std::vector<int64_t> perm1, perm2;
    std::vector<float> final_norm;
    std::vector<float> freq, sd, cd;  // infer.rs:938-962
    // weights.rs:60-76, 422-469: the probe heads the archive carries
    // (index 0 embedding, 1 confidence, 2 router).
    struct ProbeHead {
        bool present = false;
        int k = 0, q = 0, out = 0;
        std::vector<float> probes, gain, query, row_bias, proj, bias;
    } heads[3];
};


static std::vector<float> f16_tensor(const Archive& a, size_t i) {
    const Record& r = a.recs[i];
    if (r.dtype == F16) {
        std::vector<float> v(r.nbytes / 2);
        for (size_t k = 0; k < v.size(); k++) {
            uint16_t h;
            std::memcpy(&h, a.bytes(i) + 2 * k, 2);
            v[k] = f16_to_f32(h);
        }
        return v;
    }
    if (r.dtype == F32) {
        std::vector<float> v(r.nbytes / 4);
        std::memcpy(v.data(), a.bytes(i), r.nbytes);
        return v;
    }
    throw std::runtime_error("expected an f16/f32 tensor");
}

// cact.rs:620-630 (Archive::tensor): any tensor as f32 values, CQ ones
// dequantized row by row (quant.rs:259-283 = QMat::row), with its shape.
static std::vector<float> dense_tensor(const Archive& a, size_t i, std::vector<int64_t>* shape) {
    const Record& r = a.recs[i];
    if (shape) *shape = r.shape;
    if (r.dtype != CQ) return f16_tensor(a, i);
    QMat q;
    qmat_from_cq(a, i, q);
    std::vector<float> out((size_t)q.out * q.in_dim);
    for (int row = 0; row < q.out; row++) qmat_row(q, row, out.data() + (size_t)row * q.in_dim);
    return out;
}

// crates/needle-core/src/cact.rs:173-202 (Header::to_config) and
// crates/needle-engine/src/weights.rs:314-497 (record walk, fast mode),
// infer.rs:938-962 (Tables::new).
// infer.rs:938-946 (Tables::new): freq = powf(theta, i * (-2 / qk)) and
// its sine and cosine, the single-token recurrence's step.
static void rope_tables(Model& m, float theta, int qk) {
    float coef = -2.0f / (float)qk;
    m.freq.clear();
    m.sd.clear();
    m.cd.clear();
    for (int k = 0; k < qk / 2; k++) {
        float f = lpowf(theta, (float)k * coef);
        float s, co;
        lsincosf(f, &s, &co);
        m.freq.push_back(f);
        m.sd.push_back(s);
        m.cd.push_back(co);
    }
}

static void load_model(Model& m) {
    Archive a;
    parse_archive(m.bytes.data(), m.bytes.size(), a);
    Config& c = m.c;
    const uint32_t* h = a.h;
    c.vocab = h[5]; c.out_vocab = h[6]; c.d = h[7]; c.nh = h[8]; c.nkv = h[9]; c.L = h[10];
    c.qk = h[11]; c.vd = h[12]; c.max_seq = h[13]; c.hada_n = h[14]; c.lanes = h[15]; c.sw = h[16];
    c.global_mask = (uint64_t)h[17] | ((uint64_t)h[18] << 32);
    c.taps = h[19]; c.eslots = h[20]; c.esub = h[21]; c.ntables = h[22]; c.etaps = h[23]; c.edil = h[24];
    c.eseed = h[25];
    for (uint32_t i = 0; i < h[26]; i++) c.orders.push_back(h[27 + i]);
    for (uint32_t i = 0; i < h[31]; i++) c.sites.push_back(h[32 + i]);
    c.theta = bitsf(h[48]);
    c.kv_window = h[3];
    c.kv_bits = h[4];
    if (c.lanes != 4 || c.hada_n != 1024 || c.taps != 3 || c.qk != 48 || c.vd != 64 || c.etaps != 4)
        throw std::runtime_error("the native path covers the shipped geometry only");
    size_t i = 0;
    qmat_from_cq(a, i++, m.embedding);
    m.layers.resize(c.L);
    for (int l = 0; l < c.L; l++) {
        Layer& L = m.layers[l];
        L.norm_in = f16_tensor(a, i++);
        QMat q, k, v, g, o;
        qmat_from_cq(a, i++, q);
        qmat_from_cq(a, i++, k);
        qmat_from_cq(a, i++, v);
        L.q_taps = f16_tensor(a, i++);
        L.k_taps = f16_tensor(a, i++);
        L.v_taps = f16_tensor(a, i++);
        L.q_norm = f16_tensor(a, i++);
        L.k_norm = f16_tensor(a, i++);
        qmat_from_cq(a, i++, g);
        qmat_from_cq(a, i++, o);
        qmat_concat(L.qkvg, q);
        qmat_concat(L.qkvg, k);
        qmat_concat(L.qkvg, v);
        qmat_concat(L.qkvg, g);
        L.out = o;
        L.post_norm = f16_tensor(a, i++);
        L.attn_gate = f16_tensor(a, i++)[0];
        L.pre_hada = f16_tensor(a, i++);
        L.d1 = f16_tensor(a, i++);
        L.d2 = f16_tensor(a, i++);
        L.b2 = f16_tensor(a, i++);
        L.d3 = f16_tensor(a, i++);
        L.d4 = f16_tensor(a, i++);
        for (int k6 = 0; k6 < 6; k6++) L.kron[k6] = f16_tensor(a, i++);
        L.cond_v = f16_tensor(a, i++);
        L.cond_u = f16_tensor(a, i++);
    }
    int n = c.lanes;
    std::vector<float> a_pre = f16_tensor(a, i++), a_post = f16_tensor(a, i++), a_res = f16_tensor(a, i++);
    std::vector<float> b_pre = f16_tensor(a, i++), b_post = f16_tensor(a, i++), b_res = f16_tensor(a, i++);
    QMat phi[3];
    for (int k = 0; k < 3; k++) qmat_from_cq(a, i++, phi[k]);
    for (int l = 0; l < c.L; l++) {
        Layer& L = m.layers[l];
        L.a_pre = a_pre[l]; L.a_post = a_post[l]; L.a_res = a_res[l];
        L.b_pre.assign(b_pre.begin() + l * n, b_pre.begin() + (l + 1) * n);
        L.b_post.assign(b_post.begin() + l * n, b_post.begin() + (l + 1) * n);
        L.b_res.assign(b_res.begin() + l * n * n, b_res.begin() + (l + 1) * n * n);
        // weights.rs:380-391, 493: pre|post|res rows, dequantized; infer.rs:852-866 requant.
        int nc = n * c.d;
        L.phi_rows = 2 * n + n * n;
        L.phi_width = nc;
        L.phi_q.assign((size_t)L.phi_rows * nc, 0);
        L.phi_s.assign(L.phi_rows, 0.f);
        std::vector<float> row(nc);
        int k = 0;
        const int base[3] = {l * n, l * n, l * n * n};
        const int cnt[3] = {n, n, n * n};
        for (int part = 0; part < 3; part++)
            for (int rr = 0; rr < cnt[part]; rr++, k++) {
                qmat_row(phi[part], base[part] + rr, row.data());
                L.phi_s[k] = quant_i8(row.data(), nc, L.phi_q.data() + (size_t)k * nc);
            }
    }
    std::vector<float> p1 = f16_tensor(a, i++), p2 = f16_tensor(a, i++);
    for (float v : p1) m.perm1.push_back((int64_t)v);
    for (float v : p2) m.perm2.push_back((int64_t)v);
    m.engrams.resize(c.sites.size());
    for (size_t s = 0; s < c.sites.size(); s++) {
        QMat kk, vv;
        qmat_from_cq(a, i++, m.engrams[s].tables);
        qmat_from_cq(a, i++, kk);
        qmat_from_cq(a, i++, vv);
        qmat_concat(m.engrams[s].kv, kk);
        qmat_concat(m.engrams[s].kv, vv);
        m.engrams[s].taps = f16_tensor(a, i++);
    }
    m.final_norm = f16_tensor(a, i++);
    // weights.rs:422-469: probe heads between final_norm and the tokenizer.
    size_t tok_index = a.recs.size();
    for (size_t r = 0; r < a.recs.size(); r++)
        if (a.recs[r].dtype == RAW) { tok_index = r; break; }
    if (i < tok_index) {
        std::vector<float> manifest = f16_tensor(a, i++);
        const int l1 = c.L + 1;
        for (float code : manifest) {
            Model::ProbeHead h;
            std::vector<int64_t> gshape, qshape, pshape;
            h.probes = dense_tensor(a, i++, nullptr);
            h.gain = dense_tensor(a, i++, &gshape);
            h.query = dense_tensor(a, i++, &qshape);
            h.row_bias = dense_tensor(a, i++, nullptr);
            h.proj = dense_tensor(a, i++, &pshape);
            h.bias = dense_tensor(a, i++, nullptr);
            if (gshape.size() < 2 || qshape.empty() || pshape.empty()) throw std::runtime_error("probe head shapes");
            h.k = (int)gshape[1];
            h.q = (int)qshape[0];
            h.out = (int)pshape[0];
            if (h.probes.size() != (size_t)l1 * h.k * c.d) throw std::runtime_error("probe head rows do not match the depth");
            h.present = true;
            const int ci = (int)std::lround(code);
            if (ci == 3) i++;  // the router's calibration
            if (ci < 1 || ci > 3) throw std::runtime_error("unknown probe head code");
            m.heads[ci - 1] = h;
        }
    }
    if ((int)m.perm1.size() != c.hada_n || (int)m.perm2.size() != c.hada_n)
        throw std::runtime_error("Hadamard permutations do not match hada_n");
    m.site_of_layer.assign(c.L, -1);
    for (size_t s = 0; s < c.sites.size(); s++) m.site_of_layer[c.sites[s]] = (int)s;
    rope_tables(m, c.theta, c.qk);
}

// ------------------------------------------------------------- session

struct LayerState {
    std::vector<int8_t> k8;  // [slot][kvh][qk]
    std::vector<float> ks;   // [slot][kvh]
    std::vector<int8_t> v8;  // [slot][kvh][vd] (the reference keeps it transposed)
    std::vector<float> vs;   // [slot][kvh]
    std::vector<float> hist; // pre-tap q|k|v rows, newest last
};

struct RopeRow { int64_t pos; std::vector<float> c, s; };

struct Session {
    std::vector<uint32_t> tokens;
    std::vector<LayerState> layers;
    std::vector<std::vector<int8_t>> ev8;
    std::vector<std::vector<float>> evs;
    std::vector<RopeRow> rope;
    std::vector<float> last_hidden;
    std::vector<int64_t> slot_pos;
    bool has_attend = false;
    int64_t sink = 0, ring = 0;
    // infer.rs:1195-1211: with want_cells, the lane mean of the residual
    // stream of every fed position at every depth, [pos][L + 1][d].
    bool want_cells = false;
    std::vector<float> cells;
};

static Session* session_new(const Model& m) {
    Session* s = new Session();
    s->layers.resize(m.c.L);
    s->ev8.resize(m.c.sites.size());
    s->evs.resize(m.c.sites.size());
    return s;
}

// infer.rs:1749-1754
static inline int64_t slot_of(int64_t p, const Session& s) {
    if (s.has_attend && p >= s.sink) return (p - s.sink) % s.ring + s.sink;
    return p;
}

// infer.rs:1768-1776
static void mark_slots(Session& s, int64_t p0, int64_t end) {
    for (int64_t p = p0; p < end; p++) {
        int64_t sl = slot_of(p, s);
        if ((int64_t)s.slot_pos.size() <= sl) s.slot_pos.resize(sl + 1, -1);
        s.slot_pos[sl] = p;
    }
}

struct Range { int64_t a, b; };

// infer.rs:1781-1825
static std::vector<Range> key_ranges(int64_t pos, int64_t chunk_end, int window, const Session& s) {
    int64_t lo = window > 0 ? std::max<int64_t>(0, pos + 1 - window) : 0;
    std::vector<Range> coarse;
    if (!s.has_attend) {
        coarse.push_back({lo, pos + 1});
    } else {
        int64_t a_end = std::max(lo, std::min(s.sink, pos + 1));
        int64_t b0 = std::min(std::max(std::max<int64_t>(0, chunk_end - s.ring), s.sink), pos + 1);
        coarse.push_back({lo, a_end});
        coarse.push_back({b0, pos + 1});
    }
    std::vector<Range> out;
    auto push = [&](int64_t a, int64_t b) {
        if (b <= a) return;
        if (out.size() >= 16) throw std::runtime_error("too many key runs");
        out.push_back({a, b});
    };
    for (auto r : coarse) {
        if (!s.has_attend) { push(r.a, r.b); continue; }
        int64_t start = -1;
        for (int64_t p = r.a; p < r.b; p++) {
            int64_t sl = slot_of(p, s);
            bool ok = sl < (int64_t)s.slot_pos.size() && s.slot_pos[sl] == p;
            if (ok && start < 0) start = p;
            else if (!ok && start >= 0) { push(start, p); start = -1; }
        }
        if (start >= 0) push(start, r.b);
    }
    return out;
}

// infer.rs:2093-2101
void key_chunks(int64_t n, bool nested, int nkv, int64_t* count, int64_t* chunk) {
    int64_t k = nested ? 1 : std::max(1, 2 * NATIVE_TEAM / nkv);
    int64_t c = (n + 255) / 256;
    if (k * 64 <= n && c < k) c = k;
    int64_t cm = std::max<int64_t>(c, 1);
    int64_t ch = ((n + cm - 1) / cm + 15) / 16 * 16;
    *chunk = ch;
    *count = ch > 0 ? (n + ch - 1) / ch : 0;
}

// infer.rs:2222-2318 (scalar arm)
float chunk_exp(float* s, int l, float m) {
    int i = 0;
    float a[4] = {0, 0, 0, 0}, b[4] = {0, 0, 0, 0};
    while (i + 8 <= l) {
#if defined(__AVX2__)
        _mm256_storeu_ps(s + i, nexp8(_mm256_sub_ps(_mm256_loadu_ps(s + i), _mm256_set1_ps(m))));
        for (int k = 0; k < 4; k++) a[k] += s[i + k];
        for (int k = 0; k < 4; k++) b[k] += s[i + 4 + k];
#else
        for (int k = 0; k < 4; k++) { float e = nexp(s[i + k] - m); s[i + k] = e; a[k] += e; }
        for (int k = 0; k < 4; k++) { float e = nexp(s[i + 4 + k] - m); s[i + 4 + k] = e; b[k] += e; }
#endif
        i += 8;
    }
    while (i + 4 <= l) {
        for (int k = 0; k < 4; k++) { float e = nexp(s[i + k] - m); s[i + k] = e; a[k] += e; }
        i += 4;
    }
    float t[4];
    for (int k = 0; k < 4; k++) t[k] = a[k] + b[k];
    float sum = (t[0] + t[1]) + (t[2] + t[3]);
    if (l - i >= 2) {
        float e0 = lexpf(s[i] - m), e1 = lexpf(s[i + 1] - m);
        s[i] = e0;
        s[i + 1] = e1;
        sum = (e0 + sum) + e1;
        i += 2;
    }
    if (l - i == 1) {
        float e = lexpf(s[i] - m);
        s[i] = e;
        sum += e;
    }
    return sum;
}

// infer.rs:2171-2217 (scalar tail, which the SIMD arms match)
static void digits21(const float* w, int n, float qw, int8_t* hi, int8_t* mid, int8_t* lo) {
    int i = 0;
#if defined(__AVX2__)
    // eight at a time: the product and its half-away rounding as single
    // ops, the conversion truncating (a NaN or out-of-range value gives
    // INT32_MIN as cvttss2si does), the digits by arithmetic shifts and
    // masks, then narrowed to bytes by truncation
    const __m256 qv = _mm256_set1_ps(qw);
    for (; i + 8 <= n; i += 8) {
        const __m256i wq = _mm256_cvttps_epi32(round_away8(_mm256_mul_ps(_mm256_loadu_ps(w + i), qv)));
        alignas(32) int32_t h[8], md[8], l[8];
        _mm256_store_si256((__m256i*)h, _mm256_srai_epi32(wq, 14));
        _mm256_store_si256((__m256i*)md, _mm256_and_si256(_mm256_srai_epi32(wq, 7), _mm256_set1_epi32(127)));
        _mm256_store_si256((__m256i*)l, _mm256_and_si256(wq, _mm256_set1_epi32(127)));
        for (int k = 0; k < 8; k++) {
            hi[i + k] = (int8_t)h[k];
            mid[i + k] = (int8_t)md[k];
            lo[i + k] = (int8_t)l[k];
        }
    }
#endif
    for (; i < n; i++) {
        int32_t wq = (int32_t)rround(w[i] * qw);
        hi[i] = (int8_t)(wq >> 14);
        mid[i] = (int8_t)((wq >> 7) & 127);
        lo[i] = (int8_t)(wq & 127);
    }
}

struct KVView {
    const int8_t* k8; const float* ks; const int8_t* v8; const float* vs;
    int nkv, qk, vd;
};

#if defined(__AVX2__) && defined(__x86_64__)
// The P·V digit-plane sums of attend_head_ref for vd = 64 on AVX-512 VNNI:
// four keys at a time, their value rows interleaved so that each int32 holds
// one dimension's four bytes, then vpdpbusd adds digit_j * v_j over the four
// keys (digits 0..127 as unsigned bytes; exact). Int32 e of product m holds
// dimension 16 (e / 4) + 4 m + e % 4. Missing keys of the last four take
// digit 0. Adds into sh, sm, sl [64].
ORC_VNNI static void pv_sums_vnni(const KVView& kv, const int64_t* slots, int len, int kvh, const int8_t* hi, const int8_t* mid,
                                  const int8_t* lo, int32_t* sh, int32_t* sm, int32_t* sl) {
    __m512i acc[3][4];
    for (int d = 0; d < 3; d++)
        for (int m = 0; m < 4; m++) acc[d][m] = _mm512_setzero_si512();
    const int8_t* dg[3] = {hi, mid, lo};
    for (int i = 0; i < len; i += 4) {
        __m512i r[4];
        uint32_t pat[3] = {0, 0, 0};
        for (int j = 0; j < 4; j++) {
            const int key = i + j < len ? i + j : i;  // a missing key reads key i, with digit 0
            r[j] = _mm512_loadu_si512(kv.v8 + (slots[key] * kv.nkv + kvh) * 64);
            if (i + j < len)
                for (int d = 0; d < 3; d++) pat[d] |= (uint32_t)(uint8_t)dg[d][i + j] << (8 * j);
        }
        const __m512i u01l = _mm512_unpacklo_epi8(r[0], r[1]), u01h = _mm512_unpackhi_epi8(r[0], r[1]);
        const __m512i u23l = _mm512_unpacklo_epi8(r[2], r[3]), u23h = _mm512_unpackhi_epi8(r[2], r[3]);
        const __m512i w[4] = {_mm512_unpacklo_epi16(u01l, u23l), _mm512_unpackhi_epi16(u01l, u23l),
                              _mm512_unpacklo_epi16(u01h, u23h), _mm512_unpackhi_epi16(u01h, u23h)};
        for (int d = 0; d < 3; d++) {
            const __m512i p = _mm512_set1_epi32((int)pat[d]);
            for (int m = 0; m < 4; m++) acc[d][m] = _mm512_dpbusd_epi32(acc[d][m], p, w[m]);
        }
    }
    int32_t* out[3] = {sh, sm, sl};
    for (int d = 0; d < 3; d++)
        for (int m = 0; m < 4; m++) {
            alignas(64) int32_t v[16];
            _mm512_store_si512(v, acc[d][m]);
            for (int e = 0; e < 16; e++) out[d][16 * (e / 4) + 4 * m + e % 4] += v[e];
        }
}
#endif

// infer.rs:1871-2004 (attend_head_ref), with the merge of 2143-2166.
void attend_head_ref(const KVView& kv, const float* qh, int kvh, const std::vector<int64_t>& slots, bool nested, float* out) {
    const int qk = kv.qk, vd = kv.vd, nkv = kv.nkv;
    int8_t q8[64];
    float qs = quant_i8(qh, qk, q8) * INV_SQRT_QK;
    int64_t n = (int64_t)slots.size();
    int64_t count, chunk;
    key_chunks(n, nested, nkv, &count, &chunk);
    // per-thread scratch, grown to the largest chunk seen
    thread_local std::vector<float> s, scale;
    thread_local std::vector<int32_t> dots;
    thread_local std::vector<int8_t> hi, mid, lo;
    if ((int64_t)s.size() < chunk) {
        s.resize(chunk);
        scale.resize(chunk);
        dots.resize(chunk);
        hi.resize(chunk);
        mid.resize(chunk);
        lo.resize(chunk);
    }
    struct Part { float m, sum; float o[64]; };
    std::vector<Part> parts;
    parts.reserve((size_t)count);
    for (int64_t c0 = 0; c0 < n; c0 += chunk) {
        int len = (int)std::min(chunk, n - c0);
        const int64_t* sl = slots.data() + c0;
        int blocked = len / 4 * 4;
        for (int i = 0; i < len; i++) {
            dots[i] = dot_i8(q8, kv.k8 + (sl[i] * nkv + kvh) * qk, qk);
            scale[i] = kv.ks[sl[i] * nkv + kvh];
        }
        // the scores, their max, the value-scaled weights and their max:
        // eight keys at a time where the build has AVX2 (each value the same
        // single ops; a max ignores a NaN as fmax does, and the order of a
        // max changes at most the sign of a zero maximum, which no later
        // result depends on)
        int i0 = 0;
        float m = -INFINITY, wmax = 0.f;
#if defined(__AVX2__)
        __m256 mv = _mm256_set1_ps(-INFINITY);
        const __m256 qsv = _mm256_set1_ps(qs);
        for (; i0 + 8 <= blocked; i0 += 8) {
            const __m256 sc = _mm256_mul_ps(_mm256_mul_ps(_mm256_loadu_ps(scale.data() + i0),
                                                          _mm256_cvtepi32_ps(_mm256_loadu_si256((const __m256i*)(dots.data() + i0)))),
                                            qsv);
            _mm256_storeu_ps(s.data() + i0, sc);
            mv = _mm256_max_ps(sc, mv);
        }
        {
            alignas(32) float mm[8];
            _mm256_store_ps(mm, mv);
            for (int k = 0; k < 8; k++) m = rmax(m, mm[k]);
        }
#endif
        for (int i = i0; i < blocked; i++) s[i] = (scale[i] * (float)dots[i]) * qs;
        for (int i = blocked; i < len; i++) s[i] = (scale[i] * qs) * (float)dots[i];
        for (int i = i0; i < len; i++) m = rmax(m, s[i]);
        float sum = chunk_exp(s.data(), len, m);
        i0 = 0;
#if defined(__AVX2__)
        __m256 wv = _mm256_setzero_ps();
        for (; i0 + 8 <= len; i0 += 8) {
            alignas(32) float vsc[8];
            for (int k = 0; k < 8; k++) vsc[k] = kv.vs[sl[i0 + k] * nkv + kvh];
            const __m256 w = _mm256_mul_ps(_mm256_loadu_ps(s.data() + i0), _mm256_load_ps(vsc));
            _mm256_storeu_ps(s.data() + i0, w);
            wv = _mm256_max_ps(w, wv);
        }
        {
            alignas(32) float ww[8];
            _mm256_store_ps(ww, wv);
            for (int k = 0; k < 8; k++) wmax = rmax(wmax, ww[k]);
        }
#endif
        for (int i = i0; i < len; i++) {
            s[i] *= kv.vs[sl[i] * nkv + kvh];
            wmax = rmax(wmax, s[i]);
        }
        float qw = Q21 / wmax;
        digits21(s.data(), len, qw, hi.data(), mid.data(), lo.data());
        float cw = wmax * C21;
        Part p;
        p.m = m;
        p.sum = sum;
        // the three digit planes' exact integer sums, key by key
        int32_t sh[64] = {0}, sm[64] = {0}, sl2[64] = {0};
        int i_pv = 0;
#if defined(__AVX2__) && defined(__x86_64__)
        if (g_vnni && vd == 64) {
            bool nonneg = true;  // every finite weight's digits are 0..127
            for (int i = 0; i < len; i++) nonneg &= (hi[i] | mid[i] | lo[i]) >= 0;
            if (nonneg) {
                pv_sums_vnni(kv, sl, len, kvh, hi.data(), mid.data(), lo.data(), sh, sm, sl2);
                i_pv = len;
            }
        }
#endif
        for (int i = i_pv; i < len; i++) {
            const int8_t* vr = kv.v8 + (sl[i] * nkv + kvh) * vd;
            int dm = 0;
#if defined(__AVX2__)
            const __m256i h8 = _mm256_set1_epi32(hi[i]), m8 = _mm256_set1_epi32(mid[i]), l8 = _mm256_set1_epi32(lo[i]);
            for (; dm + 8 <= vd; dm += 8) {
                const __m256i v = _mm256_cvtepi8_epi32(_mm_loadl_epi64((const __m128i*)(vr + dm)));
                _mm256_storeu_si256((__m256i*)(sh + dm), _mm256_add_epi32(_mm256_loadu_si256((const __m256i*)(sh + dm)),
                                                                          _mm256_mullo_epi32(h8, v)));
                _mm256_storeu_si256((__m256i*)(sm + dm), _mm256_add_epi32(_mm256_loadu_si256((const __m256i*)(sm + dm)),
                                                                          _mm256_mullo_epi32(m8, v)));
                _mm256_storeu_si256((__m256i*)(sl2 + dm), _mm256_add_epi32(_mm256_loadu_si256((const __m256i*)(sl2 + dm)),
                                                                           _mm256_mullo_epi32(l8, v)));
            }
#endif
            for (; dm < vd; dm++) {
                sh[dm] += hi[i] * vr[dm];
                sm[dm] += mid[i] * vr[dm];
                sl2[dm] += lo[i] * vr[dm];
            }
        }
        for (int dm = 0; dm < vd; dm++)
            p.o[dm] = std::fmaf(16384.f, (float)sh[dm], std::fmaf(128.f, (float)sm[dm], (float)sl2[dm])) * cw;
        parts.push_back(p);
    }
    if (parts.size() == 1) {
        float inv = 1.0f / parts[0].sum;
        for (int dm = 0; dm < vd; dm++) out[dm] = parts[0].o[dm] * inv;
        return;
    }
    float big = -1e30f;
    for (auto& p : parts) big = rmax(big, p.m);
    float acc[64] = {0};
    float total = 0.f;
    for (auto& p : parts) {
        float w = lexpf(p.m - big);
        for (int dm = 0; dm < vd; dm++) acc[dm] = std::fmaf(p.o[dm], w, acc[dm]);
        total = std::fmaf(w, p.sum, total);
    }
    float inv = 1.0f / total;
    for (int dm = 0; dm < vd; dm++) out[dm] = acc[dm] * inv;
}

// infer.rs:1716-1744
static void rope_rows(const Model& m, Session& st, int64_t p0, int t, std::vector<float>& cos, std::vector<float>& sin) {
    int half = (int)m.freq.size();
    cos.assign((size_t)t * half, 0.f);
    sin.assign((size_t)t * half, 0.f);
    const RopeRow* prev = nullptr;
    if (!st.rope.empty() && t == 1 && st.rope.back().pos + 1 == p0) prev = &st.rope.back();
    if (prev) {
        for (int f = 0; f < half; f++) {
            cos[f] = std::fmaf(-m.sd[f], prev->s[f], m.cd[f] * prev->c[f]);
            sin[f] = std::fmaf(m.sd[f], prev->c[f], m.cd[f] * prev->s[f]);
        }
    } else {
        for (int i = 0; i < t; i++)
            for (int f = 0; f < half; f++) {
                float sv, cv;
                lsincosf(m.freq[f] * (float)(p0 + i), &sv, &cv);
                cos[(size_t)i * half + f] = cv;
                sin[(size_t)i * half + f] = sv;
            }
    }
    std::vector<RopeRow> kept;
    for (auto& r : st.rope)
        if (r.pos < p0) kept.push_back(r);
    st.rope.swap(kept);
    for (int i = 0; i < t; i++)
        st.rope.push_back({p0 + i, std::vector<float>(cos.begin() + i * half, cos.begin() + (i + 1) * half),
                           std::vector<float>(sin.begin() + i * half, sin.begin() + (i + 1) * half)});
    size_t keep = ROLLBACK + 1;
    if (st.rope.size() > 2 * keep) st.rope.erase(st.rope.begin(), st.rope.end() - keep);
}

// infer.rs:1640-1694 (scalar arm)
static void cond_weights(const float* h2, int d, const float* cond_v, float w[8]) {
    float acc[4][8] = {{0}};
    for (int j = 0; j < d; j++)
        for (int k = 0; k < 8; k++) acc[j % 4][k] = std::fmaf(h2[j], cond_v[j * 8 + k], acc[j % 4][k]);
    float lg[8], e[8];
    for (int k = 0; k < 8; k++) lg[k] = ((acc[2][k] + acc[3][k]) + acc[1][k]) + acc[0][k];
    float m = -INFINITY;
    for (int k = 0; k < 8; k++) m = rmax(m, lg[k]);
    for (int k = 0; k < 8; k++) e[k] = lexpf(lg[k] - m);
    float sum = e[7] + ((e[6] + (e[5] + e[4])) + ((e[3] + e[2]) + (e[1] + e[0])));
    float inv = 1.0f / sum;
    for (int k = 0; k < 8; k++) w[k] = e[k] * inv;
}

// infer.rs:2322-2330, 2343-2460 (scalar arm 2442-2459): T = (A^T Z) B.
// Each output is one fma chain over j = 0..31 from 0; the AVX2 form runs
// eight outputs' chains side by side (a vector fma rounds once per lane,
// as fmaf does), in the same j order.
static void kron_native(const float* z, const float* a, const float* b, float* t) {
    float mt[1024];
#if defined(__AVX2__)
    for (int c = 0; c < 32; c++) {  // mt[c][r] for r = 0..31
        __m256 o[4] = {_mm256_setzero_ps(), _mm256_setzero_ps(), _mm256_setzero_ps(), _mm256_setzero_ps()};
        for (int j = 0; j < 32; j++) {
            const __m256 zj = _mm256_set1_ps(z[j * 32 + c]);
            for (int k = 0; k < 4; k++) o[k] = _mm256_fmadd_ps(_mm256_loadu_ps(a + j * 32 + 8 * k), zj, o[k]);
        }
        for (int k = 0; k < 4; k++) _mm256_storeu_ps(mt + c * 32 + 8 * k, o[k]);
    }
    for (int r = 0; r < 32; r++) {  // t[r][c] for c = 0..31
        __m256 o[4] = {_mm256_setzero_ps(), _mm256_setzero_ps(), _mm256_setzero_ps(), _mm256_setzero_ps()};
        for (int j = 0; j < 32; j++) {
            const __m256 mj = _mm256_set1_ps(mt[j * 32 + r]);
            for (int k = 0; k < 4; k++) o[k] = _mm256_fmadd_ps(mj, _mm256_loadu_ps(b + j * 32 + 8 * k), o[k]);
        }
        for (int k = 0; k < 4; k++) _mm256_storeu_ps(t + r * 32 + 8 * k, o[k]);
    }
#else
    for (int r = 0; r < 32; r++)
        for (int c = 0; c < 32; c++) {
            float o = 0.f;
            for (int j = 0; j < 32; j++) o = std::fmaf(a[j * 32 + r], z[j * 32 + c], o);
            mt[c * 32 + r] = o;
        }
    for (int r = 0; r < 32; r++)
        for (int c = 0; c < 32; c++) {
            float o = 0.f;
            for (int j = 0; j < 32; j++) o = std::fmaf(mt[j * 32 + r], b[j * 32 + c], o);
            t[r * 32 + c] = o;
        }
#endif
}

// infer.rs:1610-1634 with axpy16 (494-528), perm_fma (689-713), silu (2463-2496)
static void mlp_native(const Model& m, const Layer& L, const float* h2, float* out) {
    const int d = m.c.d;
    float w[8];
    cond_weights(h2, d, L.cond_v.data(), w);
    float z[1024] = {0}, t[1024], cond[1024];
    for (int j = 0; j < d; j++) z[j] = h2[j] * L.d1[j];
    kron_native(z, L.kron[0].data(), L.kron[1].data(), t);
    for (int j = 0; j < 1024; j++) cond[j] = 1.0f;
    for (int k = 0; k < 8; k++)
        for (int j = 0; j < 1024; j++) cond[j] = std::fmaf(L.cond_u[k * 1024 + j], w[k], cond[j]);
    for (int j = 0; j < 1024; j++) z[j] = std::fmaf(t[m.perm1[j]], cond[j] * L.d2[j], L.b2[j]);
    silu_div(z, z, 1024);
    kron_native(z, L.kron[2].data(), L.kron[3].data(), t);
    for (int j = 0; j < 1024; j++) z[j] = t[m.perm2[j]] * L.d3[j];
    kron_native(z, L.kron[4].data(), L.kron[5].data(), t);
    for (int j = 0; j < d; j++) out[j] = t[j] * L.d4[j];
}

// infer.rs:2501-2525
static void sinkhorn64(const float z[16], float out[16]) {
    double e[16];
    for (int r = 0; r < 4; r++) {
        double m = (double)rmax(rmax(z[r * 4], z[r * 4 + 1]), rmax(z[r * 4 + 2], z[r * 4 + 3]));
        for (int c = 0; c < 4; c++) e[r * 4 + c] = lexp((double)z[r * 4 + c] - m);
    }
    for (int it = 0; it < 20; it++) {
        for (int r = 0; r < 4; r++) {
            double inv = 1.0 / ((e[r * 4] + e[r * 4 + 1]) + (e[r * 4 + 2] + e[r * 4 + 3]));
            for (int c = 0; c < 4; c++) e[r * 4 + c] *= inv;
        }
        for (int c = 0; c < 4; c++) {
            double inv = 1.0 / ((e[c] + e[4 + c]) + (e[8 + c] + e[12 + c]));
            for (int r = 0; r < 4; r++) e[r * 4 + c] *= inv;
        }
    }
    for (int k = 0; k < 16; k++) out[k] = (float)e[k];
}

// infer.rs:1707-1711
static void lane_mean(const float* x, int d, float* out) {
    for (int ch = 0; ch < d; ch++) out[ch] = (((x[ch] + x[d + ch]) + x[2 * d + ch]) + x[3 * d + ch]) * 0.25f;
}

// Named intermediate buffers recorded during a forward, for localising a
// GPU divergence (tests only).
struct Trace {
    bool on = false;
    std::map<std::string, std::vector<float>> buf;
    void put(const std::string& k, const float* p, size_t n) {
        if (on) buf[k].assign(p, p + n);
    }
};
static thread_local Trace g_trace;

// infer.rs:1244-1328
// infer.rs:1262-1272: the slot (in its table) of the n-gram of `order`
// tokens ending at position pos (tokens before position 0 read 0) for
// order index oi and head h: the seeded multiply-xor hash, folded, modulo
// the table's slots.
static uint32_t engram_slot(const uint32_t* tokens, int64_t pos, int oi, int order, int h, int stride, int slots) {
    const uint32_t SEED = 0x9E3779B9u, PRIME = 0x01000193u;  // config.rs:11-12
    uint32_t acc = SEED * (uint32_t)(oi * stride + h + 1);
    for (int j = 0; j < order; j++) {
        uint32_t tok = pos >= j ? tokens[pos - j] : 0;
        acc = (acc ^ tok) * PRIME;
    }
    acc ^= acc >> 15;
    return acc % (uint32_t)slots;
}

// infer.rs:1307-1320 with engram_tap (667-687): the dilated conv of the
// int8 value history (v8 [pos][d], vs [pos][d / 32]) at position pos, taps
// [etaps][d], into dst [d] (zeroed by the caller): tap j reads position
// pos - j * dil, stopping before position 0.
static void engram_conv_row(const float* taps, const int8_t* v8, const float* vs, int64_t pos, int etaps, int dil, int d,
                            float* dst) {
    for (int j = 0; j < etaps; j++) {
        int64_t p = pos - (int64_t)j * dil;
        if (p < 0) break;
        const int8_t* q8 = v8 + p * d;
        const float* qs = vs + p * d / 32;
        for (int ch = 0; ch < d; ch++) {
            float deq = qs[ch / 32] * (float)q8[ch];
            dst[ch] = std::fmaf(taps[(size_t)j * d + ch], deq, dst[ch]);
        }
    }
}

static void engram_native(const Model& m, Session& st, int64_t p0, int t, std::vector<std::vector<float>>& keys,
                          std::vector<std::vector<float>>& vals) {
    const Config& c = m.c;
    const int d = c.d, heads = c.eheads(), sub = c.esub;
    const int stride = c.eseed > 0 ? c.eseed : heads;
    keys.assign(c.sites.size(), {});
    vals.assign(c.sites.size(), {});
    for (size_t site = 0; site < c.sites.size(); site++) {
        std::vector<float> e((size_t)t * d, 0.f);
        for (int i = 0; i < t; i++) {
            int64_t pos = p0 + i;
            for (size_t oi = 0; oi < c.orders.size(); oi++) {
                int order = c.orders[oi];
                for (int h = 0; h < heads; h++) {
                    if (pos + 1 < order) continue;
                    int tbl = (int)oi * heads + h;
                    int row = tbl * c.eslots + (int)engram_slot(st.tokens.data(), pos, (int)oi, order, h, stride, c.eslots);
                    qmat_row(m.engrams[site].tables, row, e.data() + (size_t)i * d + tbl * sub);
                }
            }
        }
        const QMat& kvm = m.engrams[site].kv;
        QAct act = qact_new(e.data(), t, d);
        std::vector<float> kv((size_t)t * 2 * d);
        qmat_matmul(kvm, act, kv.data(), 2 * d, 0);
        auto& v8 = st.ev8[site];
        auto& vs = st.evs[site];
        v8.resize((size_t)(p0 + t) * d, 0);
        vs.resize((size_t)(p0 + t) * d / 32, 0.f);
        for (int i = 0; i < t; i++) {
            int64_t pos = p0 + i;
            for (int g = 0; g < d / 32; g++)
                vs[pos * d / 32 + g] = quant_i8(kv.data() + (size_t)i * 2 * d + d + g * 32, 32, v8.data() + pos * d + g * 32);
        }
        const std::vector<float>& taps = m.engrams[site].taps;
        std::vector<float> v((size_t)t * d, 0.f), k((size_t)t * d);
        for (int i = 0; i < t; i++) std::memcpy(&k[(size_t)i * d], &kv[(size_t)i * 2 * d], sizeof(float) * d);
        for (int i = 0; i < t; i++)
            engram_conv_row(taps.data(), v8.data(), vs.data(), p0 + i, c.etaps, c.edil, d, v.data() + (size_t)i * d);
        keys[site] = std::move(k);
        vals[site] = std::move(v);
        if (g_trace.on) {
            g_trace.put("engram_e" + std::to_string(site), e.data(), e.size());
            g_trace.put("engram_kv" + std::to_string(site), kv.data(), kv.size());
            g_trace.put("engram_v" + std::to_string(site), vals[site].data(), vals[site].size());
        }
    }
}

// infer.rs:1331-1606
// infer.rs:1359-1393 for one row: the lanes x [4 d] normalised by one rms,
// int8 (no rotation), the gate projections p [phi_rows] (int8 dots), the
// pre gates (own lane `lane`) and the block input u [d].
static void mhc_read_row(const Layer& L, int lane, const float* x, int d, float* pr, float* ur) {
    const int nc = 4 * d, ncols = L.phi_rows;
    std::vector<float> nx(nc);
    std::vector<int8_t> q8(nc);
    float r = rinv(dot16(x, x, nc), nc);
    for (int k = 0; k < nc; k++) nx[k] = x[k] * r;
    float sx = quant_i8(nx.data(), nc, q8.data());
    for (int k = 0; k < ncols; k++) {
        const int32_t acc = dot_i8(L.phi_q.data() + (size_t)k * nc, q8.data(), nc);
        pr[k] = (sx * L.phi_s[k]) * (float)acc;
    }
    float hp[4];
    for (int j = 0; j < 4; j++) {
        float off = j == lane ? 4.0f : -4.0f;
        float z = ((pr[j] * L.a_pre) + off) + L.b_pre[j];
        hp[j] = 1.0f / (lexpf(-z) + 1.0f);
    }
    for (int k = 0; k < d; k++) ur[k] = x[k] * hp[0];
    for (int b = 1; b < 4; b++)
        for (int k = 0; k < d; k++) ur[k] = std::fmaf(x[b * d + k], hp[b], ur[k]);
}

// infer.rs:1397-1418 for one row: the engram gate (when kr / vr, the site's
// key and value rows, are given) on xr in place, then the input ZC-RMSNorm
// into hr.
static void gate_norm_row(const Layer& L, float* xr, const float* kr, const float* vr, int d, float* hr) {
    if (kr) {
        float rx = rinv(dot16(xr, xr, d), d), rk = rinv(dot16(kr, kr, d), d);
        std::vector<float> a(d), b(d);
        for (int k = 0; k < d; k++) { a[k] = xr[k] * rx; b[k] = kr[k] * rk; }
        float alpha = 1.0f / (lexpf((-dot16(a.data(), b.data(), d)) / std::sqrt((float)d)) + 1.0f);
        for (int k = 0; k < d; k++) xr[k] = std::fmaf(vr[k], alpha, xr[k]);
    }
    zcn(xr, L.norm_in.data(), hr, d);
}

// infer.rs:1564-1606 for one row: o's post norm and the gated residual
// (ga: the attention gate) into x2, the pre-MLP norm, the Hadamard MLP
// (into mlp_out), the post gates (own lane `lane`) and the Sinkhorn mix of
// the gate projections pr, then the mHC write of the lanes x [4 d] in place
// from u and the old lanes.
static void post_row(const Model& m, const Layer& L, int lane, float ga, const float* o, const float* x1, const float* pr,
                     const float* ur, float* x, float* mlp_out) {
    const int d = m.c.d, n = 4, nc = n * d;
    std::vector<float> on(d), x2(d), h2(d), mlp(d);
    zcn(o, L.post_norm.data(), on.data(), d);
    for (int k = 0; k < d; k++) x2[k] = std::fmaf(on[k], ga, x1[k]);
    zcn(x2.data(), L.pre_hada.data(), h2.data(), d);
    mlp_native(m, L, h2.data(), mlp.data());
    std::memcpy(mlp_out, mlp.data(), sizeof(float) * d);
    float hpost[4];
    for (int j = 0; j < 4; j++) {
        float off = j == lane ? 0.0f : -4.0f;
        float z = ((pr[n + j] * L.a_post) + off) + L.b_post[j];
        hpost[j] = 2.0f / (lexpf(-z) + 1.0f);
    }
    float zres[16], hres[16];
    for (int k = 0; k < 16; k++) zres[k] = std::fmaf(pr[2 * n + k], L.a_res, L.b_res[k]);
    sinkhorn64(zres, hres);
    std::vector<float> old(x, x + nc);
    for (int ch = 0; ch < d; ch++) {
        float y = (x2[ch] + mlp[ch]) - ur[ch];
        for (int a = 0; a < n; a++) {
            float v = y * hpost[a];
            for (int b = 0; b < n; b++) v = std::fmaf(old[b * d + ch], hres[a * n + b], v);
            x[a * d + ch] = v;
        }
    }
}

// infer.rs:1437-1486 for one row: the three conv taps over the projection
// rows (rows[j]: the row j positions back, its q | k | v columns first;
// NULL before position 0: the tap multiplies zero), then each q and k
// head's ZC-RMSNorm and RoPE with that position's cos / sin [qk / 2]. out:
// the q | k | v row [nh qk + nkv qk + nkv vd].
static void conv_rope_row(const Layer& L, const float* const rows[3], int nh, int nkv, int qk, int vd, const float* cs,
                          const float* sn, float* out) {
    const int qd = nh * qk, kd = nkv * qk, vdim = nkv * vd, half = qk / 2;
    const struct { int start, cw; const std::vector<float>* w; } parts[3] = {
        {0, qd, &L.q_taps}, {qd, kd, &L.k_taps}, {qd + kd, vdim, &L.v_taps}};
    for (auto& pt : parts) {
        float* o = out + pt.start;
        const float* cur = rows[0] + pt.start;
        const float* w = pt.w->data();
        for (int k = 0; k < pt.cw; k++) o[k] = w[k] * cur[k];
        for (int j = 1; j < 3; j++) {
            const float* wj = w + (size_t)j * pt.cw;
            const float* r = rows[j];
            if (r) {
                for (int k = 0; k < pt.cw; k++) o[k] = std::fmaf(wj[k], r[pt.start + k], o[k]);
            } else {
                for (int k = 0; k < pt.cw; k++) o[k] = std::fmaf(wj[k], 0.0f, o[k]);
            }
        }
    }
    for (int hh = 0; hh < nh + nkv; hh++) {
        int off = hh < nh ? hh * qk : qd + (hh - nh) * qk;
        const float* scale = hh < nh ? L.q_norm.data() : L.k_norm.data();
        float* x = out + off;
        float r = rinv(dot16(x, x, qk), qk);
        for (int k = 0; k < qk; k++) {
            float tt = x[k] * r;
            x[k] = std::fmaf(tt, scale[k], tt);
        }
        for (int f = 0; f < half; f++) {
            float a = x[f], b = x[f + half];
            x[f] = std::fmaf(-sn[f], b, cs[f] * a);
            x[f + half] = std::fmaf(sn[f], a, cs[f] * b);
        }
    }
}

static void layer_native(const Model& m, int l, Session& st, int64_t p0, std::vector<float>& xs, int t,
                         const std::vector<float>& cos, const std::vector<float>& sin,
                         const std::vector<std::vector<float>>& ekeys, const std::vector<std::vector<float>>& evals) {
    const Config& c = m.c;
    const Layer& L = m.layers[l];
    const int n = c.lanes, d = c.d, nc = n * d, lane = l % n;
    const int qk = c.qk, vd = c.vd, nh = c.nh, nkv = c.nkv;
    const int qd = nh * qk, kd = nkv * qk, vdim = nkv * vd, width = qd + kd + vdim;
    const int half = qk / 2, ncols = L.phi_rows;
    const int pout = L.qkvg.out;
    std::string tag = "L" + std::to_string(l) + ".";

    // (a) mHC read
    std::vector<float> u((size_t)t * d), p((size_t)t * ncols);
    for (int i = 0; i < t; i++)
        mhc_read_row(L, lane, xs.data() + (size_t)i * nc, d, p.data() + (size_t)i * ncols, u.data() + (size_t)i * d);
    g_trace.put(tag + "u", u.data(), u.size());
    g_trace.put(tag + "p", p.data(), p.size());

    // (b) engram gate, (c) input norm, (d) A8 + qkvg
    std::vector<float> x1 = u, h((size_t)t * d);
    int site = m.site_of_layer[l];
    for (int i = 0; i < t; i++)
        gate_norm_row(L, x1.data() + (size_t)i * d, site >= 0 ? ekeys[site].data() + (size_t)i * d : nullptr,
                      site >= 0 ? evals[site].data() + (size_t)i * d : nullptr, d, h.data() + (size_t)i * d);
    g_trace.put(tag + "x1", x1.data(), x1.size());
    g_trace.put(tag + "h", h.data(), h.size());
    std::vector<float> proj((size_t)t * pout);
    {
        QAct act = qact_new(h.data(), t, d);
        qmat_matmul(L.qkvg, act, proj.data(), pout, 0);
    }
    g_trace.put(tag + "proj", proj.data(), proj.size());

    // (e) conv taps, (f) head norm + RoPE, (g) int8 KV
    LayerState& ls = st.layers[l];
    int64_t hrows = (int64_t)ls.hist.size() / width;
    std::vector<float> qkv((size_t)t * width);
    for (int i = 0; i < t; i++) {
        auto prev = [&](int j) -> const float* {
            if (j <= i) return proj.data() + (size_t)(i - j) * pout;
            if (hrows + i >= j) return ls.hist.data() + (size_t)(hrows + i - j) * width;
            return nullptr;
        };
        const float* rows[3] = {prev(0), prev(1), prev(2)};
        conv_rope_row(L, rows, nh, nkv, qk, vd, cos.data() + (size_t)i * half, sin.data() + (size_t)i * half,
                      qkv.data() + (size_t)i * width);
    }
    g_trace.put(tag + "qkv", qkv.data(), qkv.size());
    for (int i = 0; i < t; i++) ls.hist.insert(ls.hist.end(), proj.begin() + (size_t)i * pout, proj.begin() + (size_t)i * pout + width);
    {
        int64_t keep = c.taps - 1 + ROLLBACK;
        int64_t rows = (int64_t)ls.hist.size() / width;
        if (rows > 2 * keep) ls.hist.erase(ls.hist.begin(), ls.hist.begin() + (rows - keep) * width);
    }
    int64_t end = p0 + t;
    {
        int64_t need = 0;  // the largest slot the chunk writes (the ring may wrap inside it)
        for (int64_t p = p0; p < end; p++) need = std::max(need, slot_of(p, st) + 1);
        if ((int64_t)ls.ks.size() < need * nkv) {
            ls.k8.resize(need * nkv * qk, 0);
            ls.ks.resize(need * nkv, 0.f);
            ls.v8.resize(need * nkv * vd, 0);
            ls.vs.resize(need * nkv, 0.f);
        }
        for (int i = 0; i < t; i++) {
            int64_t slot = slot_of(p0 + i, st);
            const float* row = qkv.data() + (size_t)i * width;
            for (int kvh = 0; kvh < nkv; kvh++) {
                ls.ks[slot * nkv + kvh] = quant_i8(row + qd + kvh * qk, qk, ls.k8.data() + (slot * nkv + kvh) * qk);
                ls.vs[slot * nkv + kvh] = quant_i8(row + qd + kd + kvh * vd, vd, ls.v8.data() + (slot * nkv + kvh) * vd);
            }
        }
    }

    // (h) attention, (i) the gate
    std::vector<float> att((size_t)t * nh * vd);
    {
        KVView kv{ls.k8.data(), ls.ks.data(), ls.v8.data(), ls.vs.data(), nkv, qk, vd};
        int group = nh / nkv;
        bool nested = t > 1;
        int window = c.window(l);
        std::vector<std::vector<int64_t>> slots(t);
        for (int i = 0; i < t; i++) {
            int64_t pos = p0 + i;
            std::vector<Range> keys = key_ranges(pos, end, window, st);
            for (auto& r : keys)
                for (int64_t q = r.a; q < r.b; q++) slots[i].push_back(slot_of(q, st));
        }
        g_team.run(t * nh, [&](int j0, int j1) {
            for (int j = j0; j < j1; j++) {
                const int i = j / nh, hh = j % nh;
                attend_head_ref(kv, qkv.data() + (size_t)i * width + hh * qk, hh / group, slots[i], nested,
                                att.data() + ((size_t)i * nh + hh) * vd);
            }
        });
    }
    g_trace.put(tag + "attn", att.data(), att.size());
    for (int i = 0; i < t; i++) silu_div(att.data() + (size_t)i * nh * vd, proj.data() + (size_t)i * pout + width, nh * vd);
    g_trace.put(tag + "att", att.data(), att.size());

    // (j) A8 + out projection
    std::vector<float> o((size_t)t * d);
    {
        QAct act = qact_new(att.data(), t, nh * vd);
        qmat_matmul(L.out, act, o.data(), d, 0);
    }
    g_trace.put(tag + "o", o.data(), o.size());

    // (k) post block
    float ga = 1.0f / (lexpf(-L.attn_gate) + 1.0f);
    std::vector<float> mlpv((size_t)t * d);
    g_team.run(t, [&](int i0, int i1) {
        for (int i = i0; i < i1; i++)
            post_row(m, L, lane, ga, o.data() + (size_t)i * d, x1.data() + (size_t)i * d, p.data() + (size_t)i * ncols,
                     u.data() + (size_t)i * d, xs.data() + (size_t)i * nc, &mlpv[(size_t)i * d]);
    });
    g_trace.put(tag + "mlp", mlpv.data(), mlpv.size());
    g_trace.put(tag + "xs", xs.data(), xs.size());
}

enum Outputs { OUT_NONE = 0, OUT_LAST_LOGITS = 1, OUT_LAST_HIDDEN = 2, OUT_ALL_LOGITS = 3, OUT_HIDDEN = 4 };

// infer.rs:1135-1141
static void head_logits(const Model& m, const float* h, float* out) {
    QAct act = qact_new(h, 1, m.c.d);
    decode_rows(m.embedding, act, out);
}

// infer.rs:1145-1166
static void head_logits_sparse(const Model& m, const float* h, const uint32_t* ids, int n, float* out) {
    QAct act = qact_new(h, 1, m.c.d);
    for (int r = 0; r < m.c.out_rows(); r++) out[r] = NEG;
    for (int k = 0; k < n; k++) out[ids[k]] = single_row(m.embedding, (int)ids[k], act);
}

// infer.rs:1168-1240 (chunk_native; step_native computes the same for t = 1,
// crates/needle-engine/src/infer/step.rs:1-11). Returns rows written to out.
static int chunk_native(const Model& m, Session& s, const uint32_t* toks, int t, int outputs, float* out) {
    const Config& c = m.c;
    const int n = c.lanes, d = c.d, nc = n * d;
    int64_t p0 = (int64_t)s.tokens.size();
    if (p0 + t > c.max_seq) throw std::runtime_error("sequence exceeds max_seq_len");
    s.tokens.insert(s.tokens.end(), toks, toks + t);
    mark_slots(s, p0, p0 + t);
    float scale = std::sqrt((float)d);
    std::vector<float> xs((size_t)t * nc), row(d);
    for (int i = 0; i < t; i++) {
        qmat_row(m.embedding, (int)toks[i], row.data());
        for (int lane = 0; lane < n; lane++)
            for (int k = 0; k < d; k++) xs[(size_t)i * nc + lane * d + k] = row[k] * scale;
    }
    g_trace.put("embed", xs.data(), xs.size());
    const int l1 = c.L + 1;
    auto record = [&](int depth) {
        if (!s.want_cells) return;
        s.cells.resize((size_t)(p0 + t) * l1 * d);
        for (int i = 0; i < t; i++)
            lane_mean(xs.data() + (size_t)i * nc, d, s.cells.data() + ((size_t)(p0 + i) * l1 + depth) * d);
    };
    record(0);
    std::vector<std::vector<float>> ekeys, evals;
    engram_native(m, s, p0, t, ekeys, evals);
    std::vector<float> cos, sin;
    rope_rows(m, s, p0, t, cos, sin);
    g_trace.put("cos", cos.data(), cos.size());
    g_trace.put("sin", sin.data(), sin.size());
    for (int l = 0; l < c.L; l++) {
        layer_native(m, l, s, p0, xs, t, cos, sin, ekeys, evals);
        record(l + 1);
    }
    std::vector<int> rows;
    if (outputs == OUT_LAST_LOGITS || outputs == OUT_LAST_HIDDEN) rows.push_back(t - 1);
    else if (outputs == OUT_ALL_LOGITS || outputs == OUT_HIDDEN)
        for (int i = 0; i < t; i++) rows.push_back(i);
    std::vector<float> h(rows.size() * (size_t)d), mean(d);
    for (size_t r = 0; r < rows.size(); r++) {
        lane_mean(xs.data() + (size_t)rows[r] * nc, d, mean.data());
        zcn(mean.data(), m.final_norm.data(), h.data() + r * d, d);
    }
    if (!rows.empty()) s.last_hidden.assign(h.end() - d, h.end());
    g_trace.put("hidden", h.data(), h.size());
    if (outputs == OUT_NONE) return 0;
    if (outputs == OUT_LAST_HIDDEN || outputs == OUT_HIDDEN) {
        if (out) std::memcpy(out, h.data(), sizeof(float) * h.size());
        return (int)rows.size();
    }
    for (size_t r = 0; r < rows.size(); r++)
        if (out) head_logits(m, h.data() + r * d, out + r * (size_t)c.out_rows());
    return (int)rows.size();
}

// infer.rs:1105-1131: chunks of at most 32 from the feed start; the last
// chunk alone gets the outputs of a Last* request.
static int forward_native(const Model& m, Session& s, const uint32_t* ids, int n, int outputs, float* out) {
    int rows = 0;
    size_t per = (outputs == OUT_LAST_HIDDEN || outputs == OUT_HIDDEN) ? m.c.d : m.c.out_rows();
    for (int c0 = 0; c0 < n; c0 += 32) {
        int len = std::min(32, n - c0);
        bool last = c0 + len >= n;
        int want = outputs;
        if ((outputs == OUT_LAST_LOGITS || outputs == OUT_LAST_HIDDEN) && !last) want = OUT_NONE;
        rows += chunk_native(m, s, ids + c0, len, want, out ? out + rows * per : nullptr);
    }
    return rows;
}

// ------------------------------------------------------- probe heads

// linalg.rs:242-257: eight accumulators over whole groups of eight (x*y
// then +, unfused), summed (a0 + a4) + (a1 + a5) + (a2 + a6) + (a3 + a7),
// then the remainder in order.
float dot8(const float* a, const float* b, int n) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    const int chunks = n / 8;
    for (int c = 0; c < chunks; c++)
        for (int i = 0; i < 8; i++) acc[i] = acc[i] + a[c * 8 + i] * b[c * 8 + i];
    float s = (((acc[0] + acc[4]) + (acc[1] + acc[5])) + (acc[2] + acc[6])) + (acc[3] + acc[7]);
    for (int i = chunks * 8; i < n; i++) s = s + a[i] * b[i];
    return s;
}

// linalg.rs:262-277 (the reference's own constants; round half away).
float fast_exp(float x) {
    x = std::min(std::max(x, -87.33654f), 88.72283f);
    const float k = std::round(x * 1.44269504088896340736f);
    const float r = (x - k * 0.6933594f) - k * -2.1219444e-4f;
    float p = 1.9875691e-4f;
    p = p * r + 1.3981999e-3f;
    p = p * r + 8.333452e-3f;
    p = p * r + 4.1665796e-2f;
    p = p * r + 1.6666665e-1f;
    p = p * r + 5e-1f;
    const float y = ((p * r) * r + r) + 1.0f;
    return y * bitsf((uint32_t)((int32_t)k + 127) << 23);
}

// linalg.rs:309-323
static void softmax_inplace(float* x, int n) {
    float m = -INFINITY;
    for (int i = 0; i < n; i++) m = fmaxnm(m, x[i]);
    if (m == -INFINITY) {
        for (int i = 0; i < n; i++) x[i] = 0.f;
        return;
    }
    for (int i = 0; i < n; i++) x[i] = x[i] == -INFINITY ? 0.f : fast_exp(x[i] - m);
    float s = 0.f;
    for (int i = 0; i < n; i++) s = s + x[i];
    const float inv = 1.0f / s;
    for (int i = 0; i < n; i++) x[i] = x[i] * inv;
}

// linalg.rs:291-297
static void rms_unit(const float* x, int n, float* out) {
    float ss = 0.f;
    for (int i = 0; i < n; i++) ss = ss + x[i] * x[i];
    const float ms = ss / (float)n;
    const float r = 1.0f / std::sqrt(ms + 1e-6f);
    for (int i = 0; i < n; i++) out[i] = x[i] * r;
}

// heads.rs:12-56 (probe_pool) over cells [t][l1][d]: the pooled [q * d].
void probe_pool(const float* cells, int t, int l1, int d, int k, int q, const float* probes, const float* gain,
                const float* query, const float* row_bias, float* out) {
    const float inv = 1.0f / (float)std::sqrt((double)d);
    const int m = l1 * k;
    std::vector<float> r((size_t)m * d), scores(t), acc(d);
    for (int lk = 0; lk < m; lk++) {
        const int l = lk / k;
        const float* probe = probes + (size_t)lk * d;
        for (int ti = 0; ti < t; ti++) scores[ti] = dot8(cells + ((size_t)ti * l1 + l) * d, probe, d) * inv;
        softmax_inplace(scores.data(), t);
        for (int c = 0; c < d; c++) acc[c] = 0.f;
        for (int ti = 0; ti < t; ti++) {
            const float* cr = cells + ((size_t)ti * l1 + l) * d;
            for (int c = 0; c < d; c++) acc[c] = acc[c] + scores[ti] * cr[c];
        }
        float* dst = r.data() + (size_t)lk * d;
        rms_unit(acc.data(), d, dst);
        for (int c = 0; c < d; c++) dst[c] = dst[c] * gain[lk];
    }
    std::vector<float> u(m);
    for (int qi = 0; qi < q; qi++) {
        for (int j = 0; j < m; j++) u[j] = dot8(r.data() + (size_t)j * d, query + (size_t)qi * d, d) * inv + row_bias[(size_t)qi * m + j];
        softmax_inplace(u.data(), m);
        float* dst = out + (size_t)qi * d;
        for (int c = 0; c < d; c++) dst[c] = 0.f;
        for (int j = 0; j < m; j++)
            for (int c = 0; c < d; c++) dst[c] = dst[c] + u[j] * r[(size_t)j * d + c];
    }
}

// heads.rs:58-61
static void project(const Model::ProbeHead& h, const float* pooled, float* out) {
    const int n = h.q * 768;
    for (int o = 0; o < h.out; o++) out[o] = dot8(h.proj.data() + (size_t)o * n, pooled, n) + h.bias[o];
}

static void pool_head(const Model& m, const Model::ProbeHead& h, const float* cells, int t, std::vector<float>& pooled) {
    pooled.assign((size_t)h.q * m.c.d, 0.f);
    probe_pool(cells, t, m.c.L + 1, m.c.d, h.k, h.q, h.probes.data(), h.gain.data(), h.query.data(), h.row_bias.data(),
               pooled.data());
}

// heads.rs:77-90: the retrieval embedding (embedding head, else the
// confidence head's pool), unit norm. Empty without a head.
static std::vector<float> embedding_of(const Model& m, const float* cells, int t) {
    std::vector<float> v, pooled;
    if (m.heads[0].present) {
        pool_head(m, m.heads[0], cells, t, pooled);
        v.resize(m.heads[0].out);
        project(m.heads[0], pooled.data(), v.data());
    } else if (m.heads[1].present) {
        pool_head(m, m.heads[1], cells, t, v);
    } else {
        return v;
    }
    float ss = 0.f;
    for (float x : v) ss = ss + x * x;
    const float norm = std::sqrt(ss + 1e-12f);
    for (float& x : v) x = x / norm;
    return v;
}

// heads.rs:68-74
static bool confidence_of(const Model& m, const float* cells, int t, float* logit) {
    if (!m.heads[1].present) return false;
    std::vector<float> pooled, out(m.heads[1].out);
    pool_head(m, m.heads[1], cells, t, pooled);
    project(m.heads[1], pooled.data(), out.data());
    *logit = out[0];
    return true;
}

// crates/needle-engine/src/agent.rs:1114-1127: banned ids read -1e30, then the
// first index of the maximum.
static uint32_t masked_argmax(const float* x, int n, const uint8_t* allow_bits) {
    float m = -INFINITY;
    for (int i = 0; i < n; i++) {
        float v = (!allow_bits || ((allow_bits[i >> 3] >> (i & 7)) & 1)) ? x[i] : -1e30f;
        m = rmax(m, v);
    }
    for (int i = 0; i < n; i++) {
        float v = (!allow_bits || ((allow_bits[i >> 3] >> (i & 7)) & 1)) ? x[i] : -1e30f;
        if (v == m) return (uint32_t)i;
    }
    return 0;
}

// ------------------------------------------------- the call sampler (agent.rs)

// agent.rs:1130-1145: the engine's f32 exp (its own constants).
float engine_expf(float x) {
    const float LOG2E = 1.44269504088896340736f;
    x = std::min(std::max(x, -88.37626f), 88.37626f);
    float n = std::nearbyint(x * LOG2E);  // round_ties_even
    x = std::fmaf(n, -0.6933594f, x);
    x = std::fmaf(n, 2.1219444e-4f, x);
    float p = 1.9875691e-4f;
    p = std::fmaf(p, x, 1.3981999e-3f);
    p = std::fmaf(p, x, 8.333452e-3f);
    p = std::fmaf(p, x, 4.1665796e-2f);
    p = std::fmaf(p, x, 1.6666665e-1f);
    p = std::fmaf(p, x, 0.5f);
    float y = std::fmaf(x * x, p, x);
    float two_n = bitsf((uint32_t)((int32_t)n + 127) << 23);
    return std::fmaf(two_n, y, two_n);
}

// agent.rs:1241-1252 with lane_exp_sums (1147-1198, scalar arm): the max,
// then four f32 lanes of engine_expf(v - m) over whole groups of four (lane
// j takes elements 4i + j in order), summed (l0 + l1) + (l2 + l3) and
// widened, then the remainder in f64 skipping masked logits.
void softmax_stats(const float* x, int n, float* m_out, double* z_out) {
    float m = -INFINITY;
    for (int i = 0; i < n; i++) m = fmaxnm(m, x[i]);
    const int main = n / 4 * 4;
    float lanes[4] = {0.f, 0.f, 0.f, 0.f};
    for (int i = 0; i < main; i += 4)
        for (int j = 0; j < 4; j++) lanes[j] = lanes[j] + engine_expf(x[i + j] - m);
    double z = (double)((lanes[0] + lanes[1]) + (lanes[2] + lanes[3]));
    for (int i = main; i < n; i++)
        if (x[i] > -1e30f) z += lexp((double)x[i] - (double)m);
    *m_out = m;
    *z_out = z;
}

// agent.rs:335-343: the unmasked candidates (logit > -1e30) by logit, the
// lowest id first on ties; the first min(k, live) of them. Returns live.
int candidate_order(const float* x, int n, int k, int32_t* out) {
    std::vector<int32_t> order;
    for (int i = 0; i < n; i++)
        if (x[i] > -1e30f) order.push_back(i);
    const int live = (int)order.size(), head = std::min(k, live);
    std::partial_sort(order.begin(), order.begin() + head, order.end(), [&](int32_t a, int32_t b) {
        if (x[a] != x[b]) return x[a] > x[b];
        return a < b;
    });
    for (int i = 0; i < head; i++) out[i] = order[i];
    return live;
}

// ------------------------------------------------- synthetic archive writer
//
// The archive the tests and the CPU baseline load, written here from the
// reference's exporter so that the engine's own writer is checked against it
// byte for byte rather than shared by both sides.
//
// Weights: every tensor of the checkpoint is drawn ~N(0, std^2) from its own
// stream, record i (in archive order, 0-based) seeded by
// seed * 0x100000001B3 + 0x51ED270B2A6F1C3D * (i + 1): SplitMix64 words,
// uniforms (w >> 11 + 0.5) / 2^53, normals by Box-Muller in double (the
// cosine value first, then the sine one), each times std and rounded to
// f32, in the record's row-major layout. That stream is this build's own
// definition of "random init, seed 0"; everything after it follows the
// reference.

namespace {

struct SynthRng {
    uint64_t state;
    double spare = 0;
    bool have_spare = false;
    explicit SynthRng(uint64_t s) : state(s) {}
    uint64_t word() {
        state += 0x9E3779B97F4A7C15ull;
        uint64_t z = state;
        z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
        z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
        return z ^ (z >> 31);
    }
    double gauss() {
        if (have_spare) {
            have_spare = false;
            return spare;
        }
        const double u1 = ((double)(word() >> 11) + 0.5) / 9007199254740992.0;
        const double u2 = ((double)(word() >> 11) + 0.5) / 9007199254740992.0;
        const double r = std::sqrt(-2.0 * std::log(u1)), a = 6.283185307179586 * u2;
        spare = r * std::sin(a);
        have_spare = true;
        return r * std::cos(a);
    }
};

// cact.rs:254-266 (Out) with the generation recipe of its values.
struct SynthTensor {
    uint8_t dtype = 1;             // 1 f16, 2 f32, 3 CQ (cact.rs:26-31)
    std::vector<uint32_t> shape;
    uint32_t group = 0, bits = 0;
    int rows = 1, cols = 1;        // CQ: [out, d]; others: numel in cols
    std::vector<float> fixed;      // values known up front (perms, head codes)
    bool random = true;
    std::vector<uint8_t> blob;
};

// quant.rs:184-197 (pack_lsb): one row of codes LSB-first, 8 per `width`
// bytes.
void pack_lsb(const uint8_t* idx, int n, int width, uint8_t* out) {
    for (int c = 0; c < n / 8; c++) {
        uint64_t word = 0;
        for (int i = 0; i < 8; i++) word |= (uint64_t)idx[8 * c + i] << (i * width);
        for (int b = 0; b < width; b++) out[c * width + b] = (uint8_t)(word >> (8 * b));
    }
}

// quant.rs:233-256 (cq_pack) at record bits 2, 3, 4 or 5 (ternary). The
// reference packs 4-bit records only; the other widths store the nearest
// centroid of their codebook in the layout its loader reads
// (qlinear.rs:220-236, quant.rs:270-271: a ternary code c selects centroid
// c == 3 ? 0 : c + 1, so centroid k is stored as (k + 3) % 4).
void cq_pack_bits(const float* w, int rows, int d, int bits, uint8_t* packed, uint16_t* norms) {
    const std::vector<float> cb = codebook(bits, GROUP);
    const int width = code_width(bits), in_pad = (d + GROUP - 1) / GROUP * GROUP, groups = in_pad / GROUP;
    const size_t per_row = (size_t)in_pad * width / 8;
    std::vector<uint8_t> idx(in_pad);
    float g[GROUP];
    for (int r = 0; r < rows; r++) {
        const float* src = w + (size_t)r * d;
        for (int gi = 0; gi < groups; gi++) {
            const int start = gi * GROUP, take = std::min(GROUP, std::max(0, d - start));
            for (int i = 0; i < GROUP; i++) g[i] = i < take ? src[start + i] : 0.f;
            const float norm = quantize_group(g, cb.data(), (int)cb.size(), idx.data() + start);
            norms[(size_t)r * groups + gi] = f32_to_f16(norm);
        }
        if (bits == TERNARY)
            for (auto& v : idx) v = (uint8_t)((v + 3) % 4);
        pack_lsb(idx.data(), in_pad, width, packed + (size_t)r * per_row);
    }
}

}  // namespace

struct SynthSpec {
    int L = 20, vocab = 16384, slots = 18432, window = 1024, max_seq = 4096;
    uint64_t global_mask = 0, site_mask = 0, seed = 0;
    float std = 0.02f;
    std::vector<int> cq_bits;  // record bits of the i-th CQ record, 4 past the list
    unsigned heads = 0;        // bit c: probe head code c (1 embedding, 2 confidence, 3 router)
    int probes = 4, queries = 4, embedding_dim = 128;  // config.rs:27-33
};

// cact.rs:279-352 (tensors) and 362-392 (head_tensors) for the Needle 3
// geometry of config.rs:60-103 at the spec's shape knobs, then
// cact.rs:399-475 (pack) with kv_window = config.rs:452-482.
std::vector<uint8_t> synth_archive(const SynthSpec& sp) {
    const int d = 768, nh = 12, nkv = 2, qk = 48, vd = 64, lanes = 4, taps = 3, rank = 8;
    const int hn = 1024;  // config.rs:291-293: d_model's next power of two
    // config.rs:274-284 (engram_geometry): orders [2, 3], heads 768 / (2 * 128) = 3, sub_dim 128
    const int sub = 128, n_orders = 2, heads = 3, ntables = n_orders * heads;
    std::vector<int> sites;
    for (int l = 0; l < 64; l++)
        if ((sp.site_mask >> l) & 1) sites.push_back(l);
    if (sp.L < 1 || sp.L > 64) throw std::runtime_error("cact global_mask holds 64 layers");
    for (int s : sites)
        if (s >= sp.L) throw std::runtime_error("engram site outside the stack");
    if (sites.size() > 16) throw std::runtime_error("cact header holds 16 engram sites");
    std::vector<SynthTensor> ts;
    size_t n_cq = 0;
    auto row = [&](std::vector<uint32_t> shape) {
        SynthTensor t;
        t.shape = shape;
        for (auto v : shape) t.cols *= (int)v;
        ts.push_back(t);
    };
    auto cq = [&](int out, int in) {
        SynthTensor t;
        t.dtype = 3;
        t.shape = {(uint32_t)out, (uint32_t)in};
        t.rows = out;
        t.cols = in;
        t.group = GROUP;
        t.bits = (uint32_t)(n_cq < sp.cq_bits.size() ? sp.cq_bits[n_cq] : 4);
        code_width((int)t.bits);
        n_cq++;
        ts.push_back(t);
    };
    auto values = [&](uint8_t dtype, std::vector<float> v) {
        SynthTensor t;
        t.dtype = dtype;
        t.shape = {(uint32_t)v.size()};
        t.fixed = v;
        t.random = false;
        ts.push_back(t);
    };
    cq(sp.vocab, d);  // embedding/embedding
    for (int l = 0; l < sp.L; l++) {
        row({(uint32_t)d});                              // ZCRMSNorm_0/scale
        cq(nh * qk, d);                                  // q_proj
        cq(nkv * qk, d);                                 // k_proj
        cq(nkv * vd, d);                                 // v_proj
        row({(uint32_t)taps, (uint32_t)(nh * qk)});      // q_taps
        row({(uint32_t)taps, (uint32_t)(nkv * qk)});     // k_taps
        row({(uint32_t)taps, (uint32_t)(nkv * vd)});     // v_taps
        row({(uint32_t)qk});                             // q_norm
        row({(uint32_t)qk});                             // k_norm
        cq(nh * vd, d);                                  // gate_proj
        cq(d, nh * vd);                                  // out_proj
        row({(uint32_t)d});                              // post_attn_norm
        row({1});                                        // attn_gate
        row({(uint32_t)d});                              // pre_hada_norm
        for (int k = 0; k < 5; k++) row({(uint32_t)hn});  // d1 d2 b2 d3 d4
        for (int k = 0; k < 6; k++) row({32, 32});        // w1a .. w3b (config.rs hada_blocks(1024))
        row({(uint32_t)d, (uint32_t)rank});              // cond_v
        row({(uint32_t)rank, (uint32_t)hn});             // cond_u
    }
    for (int k = 0; k < 3; k++) row({(uint32_t)sp.L});                      // mhc_a_pre, _post, _res
    for (int k = 0; k < 2; k++) row({(uint32_t)sp.L, (uint32_t)lanes});     // mhc_b_pre, _post
    row({(uint32_t)sp.L, (uint32_t)(lanes * lanes)});                       // mhc_b_res
    cq(sp.L * lanes, lanes * d);                                             // mhc_phi_pre
    cq(sp.L * lanes, lanes * d);                                             // mhc_phi_post
    cq(sp.L * lanes * lanes, lanes * d);                                     // mhc_phi_res
    for (uint32_t seed : {11u, 13u}) {                                       // rng.rs:77-88 (unsplit)
        auto p = Mt19937(seed).permutation(hn);
        values(2, std::vector<float>(p.begin(), p.end()));
    }
    for (size_t s = 0; s < sites.size(); s++) {
        cq(ntables * sp.slots, sub);  // engrams_s/embedding
        cq(d, d);                     // key_proj
        cq(d, d);                     // value_proj
        row({4, (uint32_t)d});        // taps (ENGRAM_CONV_TAPS = 4)
    }
    row({(uint32_t)d});  // final_norm
    std::vector<float> codes;
    for (int c = 1; c <= 3; c++)
        if ((sp.heads >> c) & 1) codes.push_back((float)c);
    if (!codes.empty()) {
        const int l1 = sp.L + 1, k = sp.probes, q = sp.queries;
        values(1, codes);
        for (float c : codes) {
            const int out = c == 1.f ? sp.embedding_dim : c == 2.f ? 1 : 3;
            cq(l1 * k, d);                                            // probes
            row({(uint32_t)l1, (uint32_t)k});                         // gain
            cq(q, d);                                                 // query
            row({(uint32_t)q, (uint32_t)l1, (uint32_t)k});            // row_bias
            cq(out, q * d);                                           // proj kernel, transposed
            row({(uint32_t)out});                                     // proj bias
            if (c == 3.f) values(1, {0.90f, 0.00f, 0.60f});           // calibration
        }
    }
    // values and blobs (cact.rs:241-266: fp16 little-endian, f32, or CQ
    // codes followed by the f16 norms)
    std::atomic<size_t> next(0);
    auto fill = [&]() {
        for (size_t i; (i = next.fetch_add(1)) < ts.size();) {
            SynthTensor& t = ts[i];
            std::vector<float> v = t.fixed;
            if (t.random) {
                SynthRng rng(sp.seed * 0x100000001B3ull + 0x51ED270B2A6F1C3Dull * (i + 1));
                v.resize((size_t)t.rows * t.cols);
                for (auto& x : v) x = (float)(sp.std * rng.gauss());
            }
            if (t.dtype == 3) {
                const int groups = (t.cols + GROUP - 1) / GROUP;
                const size_t codes_bytes = (size_t)t.rows * groups * GROUP * code_width((int)t.bits) / 8;
                std::vector<uint16_t> norms((size_t)t.rows * groups);
                t.blob.assign(codes_bytes + norms.size() * 2, 0);
                cq_pack_bits(v.data(), t.rows, t.cols, (int)t.bits, t.blob.data(), norms.data());
                std::memcpy(t.blob.data() + codes_bytes, norms.data(), norms.size() * 2);
            } else if (t.dtype == 2) {
                t.blob.resize(v.size() * 4);
                std::memcpy(t.blob.data(), v.data(), t.blob.size());
            } else {
                t.blob.resize(v.size() * 2);
                for (size_t k = 0; k < v.size(); k++) {
                    const uint16_t h = f32_to_f16(v[k]);
                    std::memcpy(&t.blob[2 * k], &h, 2);
                }
            }
        }
    };
    {
        std::vector<std::thread> th;
        const unsigned n = std::max(1u, std::min(16u, std::thread::hardware_concurrency()));
        for (unsigned k = 0; k < n; k++) th.emplace_back(fill);
        for (auto& t : th) t.join();
    }
    // config.rs:448-482 (kv_budget_window; the config's kv_window is 0)
    const int64_t per_layer = nkv * qk + nkv * vd + (nkv * qk / 32 + nkv * vd / 32) * 4;
    const int64_t per_site = d + (d / 32) * 4, budget = 11 * 1024 * 1024 + 512 * 1024;
    int n_global = 0;
    for (int l = 0; l < sp.L; l++) n_global += (int)((sp.global_mask >> l) & 1);
    auto floor_div = [](int64_t a, int64_t b) { return a / b - ((a % b != 0) && ((a < 0) != (b < 0)) ? 1 : 0); };
    int64_t kv_window;
    if (sp.window > 0) {
        const int64_t local = std::min(sp.window, sp.max_seq);
        const int64_t fixed = ((sp.L - n_global) * per_layer + (int64_t)sites.size() * per_site) * local;
        if (n_global == 0) {
            kv_window = fixed <= budget ? sp.max_seq : std::max<int64_t>(160, local);
        } else {
            const int64_t ctx = floor_div(floor_div(budget - fixed, n_global * per_layer), 32) * 32;
            kv_window = std::max<int64_t>(160, std::min<int64_t>(ctx, sp.max_seq));
        }
    } else {
        const int64_t per_pos = sp.L * per_layer + (int64_t)sites.size() * per_site;
        kv_window = std::max<int64_t>(160, std::min<int64_t>(budget / per_pos / 32 * 32, sp.max_seq));
    }
    // cact.rs:82-119 (Header::to_bytes)
    std::vector<uint32_t> h = {TAG, (uint32_t)ts.size(), 0, (uint32_t)kv_window, 8, (uint32_t)sp.vocab, 0, d, nh, nkv,
                               (uint32_t)sp.L, qk, vd, (uint32_t)sp.max_seq, hn, lanes, (uint32_t)sp.window,
                               (uint32_t)(sp.global_mask & 0xFFFFFFFFu), (uint32_t)(sp.global_mask >> 32), taps,
                               (uint32_t)sp.slots, sub, ntables,
                               4,              // engram_conv_taps (ENGRAM_CONV_TAPS)
                               3,              // engram_conv_dilation: the largest order
                               0,              // engram_seed_heads (config.rs:85)
                               n_orders, 2, 3, 0, 0,  // the orders, padded to four
                               (uint32_t)sites.size()};
    for (int k = 0; k < 16; k++) h.push_back(k < (int)sites.size() ? (uint32_t)sites[k] : 0u);
    h.push_back(fbits(100000.0f));  // rope_theta
    std::vector<float> cbs;  // CB_BITS = [2, 3, 4] (quant.rs), each codebook(b, 128)
    for (int b : {2, 3, 4}) {
        auto c = codebook(b, GROUP);
        cbs.insert(cbs.end(), c.begin(), c.end());
    }
    h[2] = (uint32_t)cbs.size();
    if (h.size() * 4 != (size_t)HEADER_BYTES) throw std::runtime_error("header layout");
    std::vector<uint8_t> buf(HEADER_BYTES);
    std::memcpy(buf.data(), h.data(), HEADER_BYTES);
    for (float c : cbs) {
        const uint32_t u = fbits(c);
        buf.insert(buf.end(), (const uint8_t*)&u, (const uint8_t*)&u + 4);
    }
    // cact.rs:441-474: records, then 64-byte aligned blobs
    size_t pos = buf.size() + ts.size() * REC_SIZE;
    std::vector<uint64_t> offset(ts.size());
    for (size_t i = 0; i < ts.size(); i++) {
        pos = (pos + 63) / 64 * 64;
        offset[i] = pos;
        pos += ts[i].blob.size();
    }
    for (size_t i = 0; i < ts.size(); i++) {
        uint8_t r[REC_SIZE] = {};
        r[0] = ts[i].dtype;
        r[1] = (uint8_t)ts[i].shape.size();
        for (size_t k = 0; k < ts[i].shape.size() && k < 4; k++) std::memcpy(r + 4 + 4 * k, &ts[i].shape[k], 4);
        const uint64_t nbytes = ts[i].blob.size();
        std::memcpy(r + 20, &offset[i], 8);
        std::memcpy(r + 28, &nbytes, 8);
        std::memcpy(r + 36, &ts[i].group, 4);
        std::memcpy(r + 40, &ts[i].bits, 4);
        buf.insert(buf.end(), r, r + REC_SIZE);
    }
    for (size_t i = 0; i < ts.size(); i++) {
        buf.resize(offset[i], 0);
        buf.insert(buf.end(), ts[i].blob.begin(), ts[i].blob.end());
    }
    return buf;
}

}  // namespace orc

// ================================================================ C ABI

using namespace orc;

static thread_local std::string g_err;

extern "C" {

const char* orc_last_error() { return g_err.c_str(); }

uint16_t orc_f32_to_f16(float f) { return f32_to_f16(f); }
float orc_f16_to_f32(uint16_t h) { return f16_to_f32(h); }
float orc_nexp(float x) { return nexp(x); }
float orc_dot16(const float* x, const float* y, int n) { return dot16(x, y, n); }
float orc_quant_i8(const float* x, int n, int8_t* q) { return quant_i8(x, n, q); }
void orc_rotate(float* x, int n) { rotate(x, n); }
int orc_nearest(float x, const float* cb, int n) { return nearest(x, cb, n); }
int orc_codebook(int bits, int group, float* out) {
    auto v = codebook(bits, group);
    if (out) std::memcpy(out, v.data(), v.size() * 4);
    return (int)v.size();
}
void orc_mt_permutation(uint32_t seed, int n, int64_t* out) {
    Mt19937 mt(seed);
    auto p = mt.permutation(n);
    std::memcpy(out, p.data(), sizeof(int64_t) * n);
}
// rng.rs:77-88
void orc_hada_perms(int n, int split, int64_t* p1, int64_t* p2) {
    const uint32_t seeds[2] = {11, 13};
    int64_t* outs[2] = {p1, p2};
    for (int k = 0; k < 2; k++) {
        std::vector<int64_t> p;
        if (split) {
            int h = n / 2;
            p = Mt19937(seeds[k]).permutation(h);
            auto q = Mt19937(seeds[k] + 977).permutation(h);
            for (auto v : q) p.push_back(h + v);
        } else {
            p = Mt19937(seeds[k]).permutation(n);
        }
        std::memcpy(outs[k], p.data(), sizeof(int64_t) * n);
    }
}
void orc_cq_pack(const float* w, int rows, int d, uint8_t* packed, uint16_t* norms) { cq_pack(w, rows, d, packed, norms); }
float orc_prep_group(const float* x, int n, int g, int8_t* q) { return prep_group(x, n, g, q); }
float orc_chunk_exp(float* s, int l, float m) { return chunk_exp(s, l, m); }
void orc_key_chunks(int64_t n, int nested, int nkv, int64_t* count, int64_t* chunk) { key_chunks(n, nested != 0, nkv, count, chunk); }

// A raw CQ matrix of record bits `bits` (codes as stored, f16 norm bits)
// times activations x [T, in_dim]: the decode kernel when T == 1, else the
// prefill kernel with the block/remainder rule (qlinear.rs:366-419). mode 2
// = the single-row kernel per token (qlinear.rs:454-456).
int orc_cq_matmul(const uint8_t* codes, const uint16_t* norms, int out, int in_dim, int bits, const float* x, int T, int mode,
                  float* y) {
    try {
        QMat q;
        qmat_init(q, bits, out, in_dim, codes, norms);
        if (mode == 2) {
            for (int t = 0; t < T; t++) {
                QAct a = qact_new(x + (size_t)t * in_dim, 1, in_dim);
                for (int r = 0; r < out; r++) y[(size_t)t * out + r] = single_row(q, r, a);
            }
            return 0;
        }
        QAct a = qact_new(x, T, in_dim);
        qmat_matmul(q, a, y, out, 0);
        return 0;
    } catch (std::exception& e) {
        g_err = e.what();
        return -1;
    }
}

// The lane sums the matmuls use (AVX2 where the build has it) against the
// scalar loop, on n groups of weights and activations drawn from a
// seeded generator over all of int8 (both extremes forced into the
// first groups), for the 2-bit lane rule and the other one. Returns the
// groups whose four sums differ (0 when they all agree).
int orc_lane_sums_check(uint64_t seed, int n) {
    uint64_t st = seed * 0x9E3779B97F4A7C15ull + 1;
    auto next = [&]() {
        st ^= st << 13;
        st ^= st >> 7;
        st ^= st << 17;
        return st;
    };
    int bad = 0;
    int8_t w[GROUP], x[GROUP];
    for (int k = 0; k < n; k++) {
        for (int p = 0; p < GROUP; p++) {
            w[p] = (int8_t)(next() & 0xFF);
            x[p] = (int8_t)(next() & 0xFF);
            if (k == 0) w[p] = x[p] = -128;
            if (k == 1) { w[p] = -128; x[p] = 127; }
            if (k == 2) w[p] = x[p] = 127;
        }
        bool differ = false;
        for (int width : {2, 4}) {
            int32_t a[4], b[4];
            lane_sums_of(w, x, width, a);
            lane_sums_scalar(w, x, width, b);
            differ |= std::memcmp(a, b, sizeof a) != 0;
        }
#if defined(__AVX2__)
        // 4-bit codes through a codebook of sixteen int8 values: the first
        // groups' codebooks hold the extremes
        uint8_t codes[64], idx[GROUP];
        int8_t vals[16], wv[GROUP];
        for (int c = 0; c < 16; c++) vals[c] = k < 3 ? (int8_t)(c & 1 ? 127 : -128) : (int8_t)(next() & 0xFF);
        for (int b = 0; b < 64; b++) codes[b] = (uint8_t)(next() & 0xFF);
        unpack_lsb(codes, 4, GROUP, idx);
        for (int p = 0; p < GROUP; p++) wv[p] = vals[idx[p]];
        int16_t xeo[GROUP];
        for (int b0 = 0; b0 < GROUP; b0 += 32)
            for (int j = 0; j < 16; j++) {
                xeo[b0 + j] = x[b0 + 2 * j];
                xeo[b0 + 16 + j] = x[b0 + 2 * j + 1];
            }
        int32_t a[4], b[4];
        lane_sums_codes4_avx2(codes, vals, xeo, a);
        lane_sums_scalar(wv, x, 4, b);
        differ |= std::memcmp(a, b, sizeof a) != 0;
        // the byte-product form, on values without -128 (its precondition):
        // the same draws with -128 moved to -127, the extremes included
        int8_t xn[GROUP], vn[16], wn[GROUP], x8[GROUP];
        uint8_t ax[GROUP];
        for (int p = 0; p < GROUP; p++) xn[p] = x[p] == -128 ? -127 : x[p];
        for (int c = 0; c < 16; c++) vn[c] = vals[c] == -128 ? -127 : vals[c];
        for (int p = 0; p < GROUP; p++) wn[p] = vn[idx[p]];
        for (int b0 = 0; b0 < GROUP; b0 += 64)
            for (int h = 0; h < 2; h++)
                for (int j = 0; j < 16; j++)
                    for (int odd = 0; odd < 2; odd++) {
                        const int8_t v = xn[b0 + 32 * h + 2 * j + odd];
                        x8[b0 + 32 * odd + 16 * h + j] = v;
                        ax[b0 + 32 * odd + 16 * h + j] = (uint8_t)std::abs((int)v);
                    }
        _mm_storeu_si128((__m128i*)a,
                         lane_sums_codes4_ub(codes, _mm256_broadcastsi128_si256(_mm_loadu_si128((const __m128i*)vn)), x8, ax));
        lane_sums_scalar(wn, xn, 4, b);
        differ |= std::memcmp(a, b, sizeof a) != 0;
#if defined(__x86_64__)
        if (g_vnni) {  // the VNNI form over all of int8 (no -128 restriction)
            uint8_t vb[16];
            for (int c = 0; c < 16; c++) vb[c] = (uint8_t)(vals[c] + 128);
            int8_t x8v[GROUP];
            int32_t sumx[4] = {0, 0, 0, 0};
            for (int p = 0; p < GROUP; p++) {
                x8v[(p & 1) * 64 + p / 2] = x[p];
                sumx[(p % 32) / 8] += x[p];
            }
            lane_sums_vnni(codes, vb, x8v, sumx, a);
            lane_sums_scalar(wv, x, 4, b);
            differ |= std::memcmp(a, b, sizeof a) != 0;
        }
#endif
#endif
        bad += differ;
    }
    return bad;
}

// silu_div (vectorised where the build has AVX2) against the scalar
// x / (nexp(-g) + 1) on n values from a seeded generator spread over the
// clamp range and past it, plus the specials (zeros, infinities, NaN, the
// clamp bounds, halfway points of the rounding). Returns the values whose
// bits differ. Signalling NaNs are left out of the raw-bit draws: no
// arithmetic produces one, and glibc's fmaxf turns one into NaN where the
// vector max (as CUDA's fmaxf) takes the bound.
int orc_nexp_check(uint64_t seed, int n) {
    uint64_t st = seed * 0x9E3779B97F4A7C15ull + 1;
    auto next = [&]() {
        st ^= st << 13;
        st ^= st >> 7;
        st ^= st << 17;
        return st;
    };
    std::vector<float> g;
    const float specials[] = {0.f, -0.f, INFINITY, -INFINITY, NAN, bitsf(0xc2b0c0a5u), bitsf(0x42b0c0a5u), 88.8f, -88.8f,
                              0.5f * 0.6931472f, -0.5f * 0.6931472f, 1e-30f, -1e-30f, 1.5f * 0.6931472f};
    for (float v : specials) g.push_back(v);
    while ((int)g.size() < n) {
        const uint64_t u = next();
        g.push_back(((float)(u >> 40) / (float)(1u << 24) - 0.5f) * 240.f);  // [-120, 120)
        uint32_t b = (uint32_t)u;
        if ((b & 0x7f800000u) == 0x7f800000u && (b & 0x007fffffu)) b |= 0x00400000u;  // NaNs quiet
        g.push_back(bitsf(b));                                                         // any other bits
    }
    std::vector<float> x(g.size()), a(g.size());
    for (size_t i = 0; i < g.size(); i++) x[i] = a[i] = bitsf((uint32_t)(next() >> 7) & 0x3fffffffu);
    silu_div(a.data(), g.data(), (int64_t)g.size());
    int bad = 0;
    for (size_t i = 0; i < g.size(); i++) {
        const float b = x[i] / (nexp(-g[i]) + 1.0f);
        bad += fbits(a[i]) != fbits(b) && !(a[i] != a[i] && b != b);
    }
    return bad;
}

// quant_i8 (vectorised where the build has AVX2) against the scalar loop
// on n rows of seeded values (row lengths 1-200, magnitudes from 1e-40 to
// 1e30, infinities, quiet NaNs, zeros), and the vector rounding against
// std::round on exact halves and raw bits. Returns the mismatches.
int orc_quant_check(uint64_t seed, int n) {
    uint64_t st = seed * 0x9E3779B97F4A7C15ull + 1;
    auto next = [&]() {
        st ^= st << 13;
        st ^= st >> 7;
        st ^= st << 17;
        return st;
    };
    int bad = 0;
    std::vector<float> x(200);
    std::vector<int8_t> a(200), b(200);
    for (int k = 0; k < n; k++) {
        const int len = 1 + (int)(next() % 200);
        const float scale = std::ldexp(1.0f, (int)(next() % 230) - 133);
        for (int i = 0; i < len; i++) {
            const uint64_t u = next();
            float v = ((float)(u >> 40) / (float)(1u << 24) - 0.5f) * scale;
            if (u % 97 == 0) v = (u & 1) ? INFINITY : -INFINITY;
            if (u % 89 == 0) v = 0.f;
            if (k % 50 == 0 && u % 83 == 0) v = NAN;
            x[i] = v;
        }
        const float s1 = quant_i8(x.data(), len, a.data()), s2 = quant_i8_scalar(x.data(), len, b.data());
        bad += fbits(s1) != fbits(s2) || std::memcmp(a.data(), b.data(), len) != 0;
    }
#if defined(__AVX2__)
    for (int k = 0; k < n; k++) {
        alignas(32) float v[8], r[8];
        for (int j = 0; j < 8; j++) {
            const uint64_t u = next();
            uint32_t bits = (uint32_t)u;
            if ((bits & 0x7f800000u) == 0x7f800000u) bits &= 0xff800000u;  // infinities, no NaNs
            v[j] = (j & 1) ? bitsf(bits) : ((float)(int)(u % 2001) - 1000.f) * 0.5f;  // exact halves
        }
        _mm256_store_ps(r, round_away8(_mm256_load_ps(v)));
        for (int j = 0; j < 8; j++) bad += fbits(r[j]) != fbits(std::round(v[j]));
    }
#endif
    return bad;
}

// The team one sequence's forward splits its matmul rows, attention heads
// and post-block rows over (1: the calling thread alone). Not to be called
// while a forward runs.
void orc_set_team(int threads) { g_team.resize(std::max(1, std::min(threads, 256))); }

// Resizes the team and runs small jobs on it `rounds` times in quick
// succession (a job right after each resize included); returns the jobs
// whose sum came out wrong. The team is left at one thread.
int orc_team_stress(int rounds) {
    int bad = 0;
    for (int k = 0; k < rounds; k++) {
        g_team.resize(2 + k % 7);
        for (int j = 0; j < 4; j++) {
            const int items = 1 + (k * 7 + j * 13) % 200;
            std::vector<int> hit(items, 0);
            g_team.run(items, [&](int i0, int i1) {
                for (int i = i0; i < i1; i++) hit[i]++;
            });
            for (int i = 0; i < items; i++) bad += hit[i] != 1;
        }
        // a slice that throws: every other slice still runs, and the
        // caller gets the exception
        const int items = 64;
        std::vector<int> hit(items, 0);
        bool caught = false;
        try {
            g_team.run(items, [&](int i0, int i1) {
                for (int i = i0; i < i1; i++) hit[i]++;
                if (i0 == 0) throw std::runtime_error("slice 0");
            });
        } catch (const std::runtime_error&) {
            caught = true;
        }
        bad += !caught;
        for (int i = 0; i < items; i++) bad += hit[i] != 1;
    }
    g_team.resize(1);
    return bad;
}
int orc_team_size() { return g_team.size(); }

// fwht on 128 points (vectorised where the build has AVX2) against the
// scalar butterflies, bit for bit, on n seeded vectors (raw bits without
// signalling NaNs, and ordinary values). Returns the vectors that differ.
int orc_fwht_check(uint64_t seed, int n) {
    uint64_t st = seed * 0x9E3779B97F4A7C15ull + 1;
    auto next = [&]() {
        st ^= st << 13;
        st ^= st >> 7;
        st ^= st << 17;
        return st;
    };
    int bad = 0;
    for (int k = 0; k < n; k++) {
        float a[128], b[128];
        for (int i = 0; i < 128; i++) {
            uint32_t u = (uint32_t)next();
            if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x007fffffu)) u |= 0x00400000u;
            a[i] = b[i] = (k % 2) ? bitsf(u) : ((float)(int)(u % 20001) - 10000.f) * 1e-3f;
        }
        fwht(a, 128);
        fwht_scalar(b, 128);
        for (int i = 0; i < 128; i++)
            if (fbits(a[i]) != fbits(b[i]) && !(a[i] != a[i] && b[i] != b[i])) {
                bad++;
                break;
            }
    }
    return bad;
}

// infer.rs:1610-1634 (mlp_native) on one pre-MLP row h2 [d] with the
// layer's MLP weights given directly (values of f16 weights as floats):
// d1, d4 [d]; d2, b2, d3 [1024]; kron [6][1024]; cond_v [d][8];
// cond_u [8][1024]; perm1, perm2 [1024]. out [d].
int orc_mlp(const float* h2, int d, const float* d1, const float* d2, const float* b2, const float* d3, const float* d4,
            const float* kron, const float* cond_v, const float* cond_u, const int64_t* perm1, const int64_t* perm2,
            float* out) {
    if (d < 1 || d > 1024) return -1;
    Model m;
    m.c.d = d;
    m.perm1.assign(perm1, perm1 + 1024);
    m.perm2.assign(perm2, perm2 + 1024);
    for (int j = 0; j < 1024; j++)
        if (m.perm1[j] < 0 || m.perm1[j] >= 1024 || m.perm2[j] < 0 || m.perm2[j] >= 1024) return -1;
    Layer L;
    L.d1.assign(d1, d1 + d);
    L.d4.assign(d4, d4 + d);
    L.d2.assign(d2, d2 + 1024);
    L.b2.assign(b2, b2 + 1024);
    L.d3.assign(d3, d3 + 1024);
    for (int k = 0; k < 6; k++) L.kron[k].assign(kron + k * 1024, kron + (k + 1) * 1024);
    L.cond_v.assign(cond_v, cond_v + (size_t)d * 8);
    L.cond_u.assign(cond_u, cond_u + 8 * 1024);
    mlp_native(m, L, h2, out);
    return 0;
}

// infer.rs:1359-1418 on one row with given weights: the mHC read of the
// lanes x [4 d] (gate rows phi_q [24][4 d] int8 with scales phi_s [24],
// a_pre, b_pre [4], own lane `lane`) into p [24] and u [d]; then the engram
// gate with the site's key / value rows kr, vr [d] (both NULL: no site) and
// the input norm (norm_in [d]) into x1 [d] and h [d].
int orc_mhc_read(const float* x, int d, const int8_t* phi_q, const float* phi_s, float a_pre, const float* b_pre, int lane,
                 const float* kr, const float* vr, const float* norm_in, float* p, float* u, float* x1, float* h) {
    if (d < 16 || d % 16 || lane < 0 || lane > 3 || (!kr) != (!vr)) return -1;
    Layer L;
    L.phi_rows = 24;
    L.phi_width = 4 * d;
    L.phi_q.assign(phi_q, phi_q + (size_t)24 * 4 * d);
    L.phi_s.assign(phi_s, phi_s + 24);
    L.a_pre = a_pre;
    L.b_pre.assign(b_pre, b_pre + 4);
    L.norm_in.assign(norm_in, norm_in + d);
    mhc_read_row(L, lane, x, d, p, u);
    std::memcpy(x1, u, sizeof(float) * d);
    gate_norm_row(L, x1, kr, vr, d, h);
    return 0;
}

// infer.rs:1564-1606 on one row with given weights: post_norm, pre_hada
// [d], attn_gate, a_post, b_post [4], a_res, b_res [16], the MLP weights as
// orc_mlp takes them, own lane `lane`; o, x1, u [d] and the gate
// projections pr [24]; the lanes x [4 d] updated in place, mlp_out [d].
int orc_post_row(int d, const float* post_norm, const float* pre_hada, float attn_gate, float a_post, const float* b_post,
                 float a_res, const float* b_res, const float* d1, const float* d2, const float* b2, const float* d3,
                 const float* d4, const float* kron, const float* cond_v, const float* cond_u, const int64_t* perm1,
                 const int64_t* perm2, int lane, const float* o, const float* x1, const float* pr, const float* u, float* x,
                 float* mlp_out) {
    if (d < 16 || d % 16 || d > 1024 || lane < 0 || lane > 3) return -1;
    Model m;
    m.c.d = d;
    m.perm1.assign(perm1, perm1 + 1024);
    m.perm2.assign(perm2, perm2 + 1024);
    for (int j = 0; j < 1024; j++)
        if (m.perm1[j] < 0 || m.perm1[j] >= 1024 || m.perm2[j] < 0 || m.perm2[j] >= 1024) return -1;
    Layer L;
    L.post_norm.assign(post_norm, post_norm + d);
    L.pre_hada.assign(pre_hada, pre_hada + d);
    L.attn_gate = attn_gate;
    L.a_post = a_post;
    L.b_post.assign(b_post, b_post + 4);
    L.a_res = a_res;
    L.b_res.assign(b_res, b_res + 16);
    L.d1.assign(d1, d1 + d);
    L.d4.assign(d4, d4 + d);
    L.d2.assign(d2, d2 + 1024);
    L.b2.assign(b2, b2 + 1024);
    L.d3.assign(d3, d3 + 1024);
    for (int k = 0; k < 6; k++) L.kron[k].assign(kron + k * 1024, kron + (k + 1) * 1024);
    L.cond_v.assign(cond_v, cond_v + (size_t)d * 8);
    L.cond_u.assign(cond_u, cond_u + 8 * 1024);
    const float ga = 1.0f / (lexpf(-L.attn_gate) + 1.0f);
    post_row(m, L, lane, ga, o, x1, pr, u, x, mlp_out);
    return 0;
}

// infer.rs:1437-1486 on one row with given weights (the Needle 3 heads: 12
// q and 2 kv heads of 48, values 64): rows cur, prev1, prev2 [800] (prev
// NULL before position 0), taps q_taps [3][576], k_taps [3][96], v_taps
// [3][128], q_norm, k_norm [48], cos / sin [24]. out [800].
int orc_conv_rope(const float* cur, const float* prev1, const float* prev2, const float* q_taps, const float* k_taps,
                  const float* v_taps, const float* q_norm, const float* k_norm, const float* cs, const float* sn, float* out) {
    if (!cur || (!prev1 && prev2)) return -1;
    Layer L;
    L.q_taps.assign(q_taps, q_taps + 3 * 576);
    L.k_taps.assign(k_taps, k_taps + 3 * 96);
    L.v_taps.assign(v_taps, v_taps + 3 * 128);
    L.q_norm.assign(q_norm, q_norm + 48);
    L.k_norm.assign(k_norm, k_norm + 48);
    const float* rows[3] = {cur, prev1, prev2};
    conv_rope_row(L, rows, 12, 2, 48, 64, cs, sn, out);
    return 0;
}

// infer.rs:1716-1744 (rope_rows) for a session that fed positions
// p0 - n_prev .. p0 - 1 one row at a time before, then asks for t rows
// from p0: each of those calls and this one as the oracle's sessions make
// them (the direct angles for a chunk, the recurrence for a single token
// after the newest row). Writes this call's cos / sin [t][qk / 2].
int orc_rope_rows(float theta, int qk, int64_t p0, int n_prev, int t, float* cos_out, float* sin_out) {
    if (qk < 2 || qk % 2 || t < 1 || n_prev < 0 || n_prev > p0) return -1;
    Model m;
    rope_tables(m, theta, qk);
    Session st;
    std::vector<float> cs, sn;
    if (n_prev > 0) rope_rows(m, st, p0 - n_prev, 1, cs, sn);  // the first as a direct row
    for (int64_t p = p0 - n_prev + 1; p < p0; p++) rope_rows(m, st, p, 1, cs, sn);
    rope_rows(m, st, p0, t, cs, sn);
    std::memcpy(cos_out, cs.data(), sizeof(float) * cs.size());
    std::memcpy(sin_out, sn.data(), sizeof(float) * sn.size());
    return 0;
}

// The engram slot of each (position, order index, head) for tokens [n]
// (orders [n_orders], heads, seed stride, slots): out [n][n_orders][heads],
// -1 where the position is shorter than the order.
void orc_engram_slots(const uint32_t* tokens, int n, const int* orders, int n_orders, int heads, int stride, int slots,
                      int64_t* out) {
    for (int pos = 0; pos < n; pos++)
        for (int oi = 0; oi < n_orders; oi++)
            for (int h = 0; h < heads; h++)
                out[((size_t)pos * n_orders + oi) * heads + h] =
                    pos + 1 < orders[oi] ? -1 : (int64_t)engram_slot(tokens, pos, oi, orders[oi], h, stride, slots);
}

// engram_conv_row at position pos over the history v8 [pos + 1][d], vs
// [pos + 1][d / 32] with taps [etaps][d]: out [d].
void orc_engram_conv(const float* taps, const int8_t* v8, const float* vs, int64_t pos, int etaps, int dil, int d, float* out) {
    std::fill(out, out + d, 0.f);
    engram_conv_row(taps, v8, vs, pos, etaps, dil, d, out);
}

// 1 when the 4-bit matmuls run their lane sums on AVX-512 VNNI.
int orc_vnni() { return g_vnni ? 1 : 0; }

// The attention's P·V digit-plane sums on VNNI (where the host has it)
// against the plain key loop: n cases of 1-300 keys in shuffled slots of a
// two-head cache, values over all of int8, digits 0..127. Returns the cases
// whose sums differ (0 also where there is no VNNI form to check).
int orc_pv_check(uint64_t seed, int n) {
    int bad = 0;
#if defined(__AVX2__) && defined(__x86_64__)
    if (!g_vnni) return 0;
    uint64_t st = seed * 0x9E3779B97F4A7C15ull + 1;
    auto next = [&]() {
        st ^= st << 13;
        st ^= st >> 7;
        st ^= st << 17;
        return st;
    };
    for (int k = 0; k < n; k++) {
        const int len = 1 + (int)(next() % 300), cap = len + 7, nkv = 2, kvh = (int)(next() & 1);
        std::vector<int8_t> v8((size_t)cap * nkv * 64), hi(len), mid(len), lo(len);
        for (auto& v : v8) v = (int8_t)(next() & 0xFF);
        if (k == 0) std::fill(v8.begin(), v8.end(), (int8_t)-128);
        std::vector<int64_t> slots(cap);
        for (int i = 0; i < cap; i++) slots[i] = i;
        for (int i = cap - 1; i > 0; i--) std::swap(slots[i], slots[next() % (i + 1)]);
        slots.resize(len);
        for (int i = 0; i < len; i++) {
            hi[i] = (int8_t)(k == 0 ? 127 : next() % 128);
            mid[i] = (int8_t)(next() % 128);
            lo[i] = (int8_t)(next() % 128);
        }
        KVView kv{nullptr, nullptr, v8.data(), nullptr, nkv, 48, 64};
        int32_t a[3][64] = {{0}}, b[3][64] = {{0}};
        pv_sums_vnni(kv, slots.data(), len, kvh, hi.data(), mid.data(), lo.data(), a[0], a[1], a[2]);
        for (int i = 0; i < len; i++) {
            const int8_t* vr = v8.data() + (slots[i] * nkv + kvh) * 64;
            for (int dm = 0; dm < 64; dm++) {
                b[0][dm] += hi[i] * vr[dm];
                b[1][dm] += mid[i] * vr[dm];
                b[2][dm] += lo[i] * vr[dm];
            }
        }
        bad += std::memcmp(a, b, sizeof a) != 0;
    }
#else
    (void)seed;
    (void)n;
#endif
    return bad;
}

// QMat::row of a raw CQ matrix of record bits `bits` (qlinear.rs:309-323).
int orc_cq_row(const uint8_t* codes, const uint16_t* norms, int rows, int in_dim, int bits, int r, float* out) {
    try {
        const int groups = (in_dim + GROUP - 1) / GROUP;
        const size_t bpr = (size_t)groups * 16 * code_width(bits);
        QMat q;
        qmat_init(q, bits, 1, in_dim, codes + (size_t)r * bpr, norms + (size_t)r * groups);
        qmat_row(q, 0, out);
        (void)rows;
        return 0;
    } catch (std::exception& e) {
        g_err = e.what();
        return -1;
    }
}

// attend_head_ref over caller-provided caches ([slot][kvh][qk] keys,
// [slot][kvh][vd] values) and a slot list.
void orc_attend_head(const int8_t* k8, const float* ks, const int8_t* v8, const float* vs, int nkv, int qk, int vd,
                     const float* qh, int kvh, const int64_t* slots, int n, int nested, float* out) {
    KVView kv{k8, ks, v8, vs, nkv, qk, vd};
    std::vector<int64_t> sl(slots, slots + n);
    attend_head_ref(kv, qh, kvh, sl, nested != 0, out);
}

// ---- model level

void* orc_model_load(const uint8_t* bytes, uint64_t n) {
    try {
        Model* m = new Model();
        m->bytes.assign(bytes, bytes + n);
        load_model(*m);
        m->bytes.clear();
        m->bytes.shrink_to_fit();
        return m;
    } catch (std::exception& e) {
        g_err = e.what();
        return nullptr;
    }
}
void orc_model_free(void* m) { delete (Model*)m; }
int orc_model_dims(void* mp, int* out) {
    Model* m = (Model*)mp;
    out[0] = m->c.vocab; out[1] = m->c.out_rows(); out[2] = m->c.d; out[3] = m->c.L;
    out[4] = m->c.nh; out[5] = m->c.nkv; out[6] = m->c.qk; out[7] = m->c.vd; out[8] = m->c.max_seq;
    return 0;
}
void* orc_session_new(void* m) { return session_new(*(Model*)m); }
void orc_session_free(void* s) { delete (Session*)s; }
void* orc_session_clone(void* s) { return new Session(*(Session*)s); }
int orc_session_len(void* s) { return (int)((Session*)s)->tokens.size(); }
// model.rs:81-113 + infer.rs:1055-1077 (Session::rollback): drop the last
// n <= ROLLBACK positions without recomputing: the conv history loses its
// last n rows, the engram history and RoPE rows their dropped positions;
// KV slots and the slot map stay.
int orc_session_rollback(void* mp, void* sp, int64_t n) {
    try {
        const Model& m = *(const Model*)mp;
        Session& s = *(Session*)sp;
        if (n > ROLLBACK) throw std::runtime_error("rollback exceeds ROLLBACK");
        if (n > (int64_t)s.tokens.size()) throw std::runtime_error("rollback past the start");
        if (n == 0) return 0;
        const int64_t len = (int64_t)s.tokens.size() - n;
        s.tokens.resize(len);
        const int64_t width = (int64_t)(m.c.nh + m.c.nkv) * m.c.qk + (int64_t)m.c.nkv * m.c.vd;
        for (auto& ls : s.layers) {
            const int64_t rows = (int64_t)ls.hist.size() / width;
            ls.hist.resize((size_t)std::max<int64_t>(0, rows - n) * width);
        }
        for (size_t site = 0; site < s.ev8.size(); site++) {
            if ((int64_t)s.ev8[site].size() > len * m.c.d) s.ev8[site].resize((size_t)len * m.c.d);
            if ((int64_t)s.evs[site].size() > len * m.c.d / 32) s.evs[site].resize((size_t)len * m.c.d / 32);
        }
        std::vector<RopeRow> kept;
        for (auto& r : s.rope)
            if (r.pos < len) kept.push_back(r);
        s.rope.swap(kept);
        return 0;
    } catch (std::exception& e) {
        g_err = e.what();
        return -1;
    }
}

// model.rs:116-126 + infer.rs:1039-1053 (Session::rewind_zeroed): forget
// positions len..: the conv history is emptied, the engram history
// truncated, the RoPE rows dropped; KV slots and slot map stay.
int orc_session_rewind_zeroed(void* mp, void* sp, int64_t len) {
    const Model& m = *(const Model*)mp;
    Session& s = *(Session*)sp;
    if (len < (int64_t)s.tokens.size()) s.tokens.resize(len);
    for (auto& ls : s.layers) ls.hist.clear();
    for (size_t site = 0; site < s.ev8.size(); site++) {
        if ((int64_t)s.ev8[site].size() > len * m.c.d) s.ev8[site].resize((size_t)len * m.c.d);
        if ((int64_t)s.evs[site].size() > len * m.c.d / 32) s.evs[site].resize((size_t)len * m.c.d / 32);
    }
    s.rope.clear();
    return 0;
}

// model.rs:128-145 (Session::truncate): up to ROLLBACK positions by
// rollback, more by a fresh session (no attention span) fed the first len
// tokens.
int orc_session_truncate(void* mp, void* sp, int64_t len) {
    try {
        const Model& m = *(const Model*)mp;
        Session& s = *(Session*)sp;
        const int64_t have = (int64_t)s.tokens.size();
        if (len >= have) return 0;
        if (have - len <= ROLLBACK) return orc_session_rollback(mp, sp, have - len);
        std::vector<uint32_t> toks(s.tokens.begin(), s.tokens.begin() + len);
        std::unique_ptr<Session> fresh(session_new(m));
        s = *fresh;
        if (len > 0) forward_native(m, s, toks.data(), (int)len, OUT_NONE, nullptr);
        return 0;
    } catch (std::exception& e) {
        g_err = e.what();
        return -1;
    }
}

void orc_session_set_attend(void* s, int64_t sink, int64_t ring) {
    Session* ss = (Session*)s;
    ss->has_attend = ring > 0;
    ss->sink = sink;
    ss->ring = ring;
}

int orc_forward(void* m, void* s, const uint32_t* ids, int n, int outputs, float* out) {
    try {
        return forward_native(*(Model*)m, *(Session*)s, ids, n, outputs, out);
    } catch (std::exception& e) {
        g_err = e.what();
        return -1;
    }
}

void orc_head_logits(void* m, const float* h, float* out) { head_logits(*(Model*)m, h, out); }
void orc_head_logits_sparse(void* m, const float* h, const uint32_t* ids, int n, float* out) {
    head_logits_sparse(*(Model*)m, h, ids, n, out);
}
int orc_last_hidden(void* s, float* out) {
    Session* ss = (Session*)s;
    if (out) std::memcpy(out, ss->last_hidden.data(), ss->last_hidden.size() * 4);
    return (int)ss->last_hidden.size();
}
uint32_t orc_masked_argmax(const float* x, int n, const uint8_t* allow_bits) { return masked_argmax(x, n, allow_bits); }
float orc_engine_expf(float x) { return engine_expf(x); }
float orc_fast_exp(float x) { return fast_exp(x); }
float orc_dot8(const float* a, const float* b, int n) { return dot8(a, b, n); }
void orc_probe_pool(const float* cells, int t, int l1, int d, int k, int q, const float* probes, const float* gain,
                    const float* query, const float* row_bias, float* out) {
    probe_pool(cells, t, l1, d, k, q, probes, gain, query, row_bias, out);
}
int orc_head_present(void* mp, int code) {
    Model& m = *(Model*)mp;
    return code >= 1 && code <= 3 && m.heads[code - 1].present ? 1 : 0;
}
// heads.rs:63-66 + 77-90 (needle_embed's computation over token ids): a
// fresh session fed `ids` in chunks of 32 with cells, then the embedding.
// Returns its width (out == NULL: only the width), -1 without a head.
int orc_embed(void* mp, const uint32_t* ids, int n, float* out) {
    try {
        Model& m = *(Model*)mp;
        if (!m.heads[0].present && !m.heads[1].present) throw std::runtime_error("this archive carries no probe head");
        const int dim = m.heads[0].present ? m.heads[0].out : m.heads[1].q * m.c.d;
        if (!out) return dim;
        std::unique_ptr<Session> s(session_new(m));
        s->want_cells = true;
        forward_native(m, *s, ids, n, OUT_NONE, nullptr);
        std::vector<float> v = embedding_of(m, s->cells.data(), n);
        std::memcpy(out, v.data(), sizeof(float) * v.size());
        return dim;
    } catch (std::exception& e) {
        g_err = e.what();
        return -1;
    }
}
// heads.rs:68-74: the confidence head's logit for `ids`.
int orc_confidence(void* mp, const uint32_t* ids, int n, float* out) {
    try {
        Model& m = *(Model*)mp;
        std::unique_ptr<Session> s(session_new(m));
        s->want_cells = true;
        forward_native(m, *s, ids, n, OUT_NONE, nullptr);
        if (!confidence_of(m, s->cells.data(), n, out)) throw std::runtime_error("this archive carries no confidence head");
        return 0;
    } catch (std::exception& e) {
        g_err = e.what();
        return -1;
    }
}
// The cells [n][L + 1][d] of a fresh session fed `ids`.
int orc_cells(void* mp, const uint32_t* ids, int n, float* out) {
    try {
        Model& m = *(Model*)mp;
        std::unique_ptr<Session> s(session_new(m));
        s->want_cells = true;
        forward_native(m, *s, ids, n, OUT_NONE, nullptr);
        std::memcpy(out, s->cells.data(), sizeof(float) * s->cells.size());
        return 0;
    } catch (std::exception& e) {
        g_err = e.what();
        return -1;
    }
}
void orc_softmax_stats(const float* x, int n, float* m, double* z) { softmax_stats(x, n, m, z); }
int orc_candidate_order(const float* x, int n, int k, int32_t* out) { return candidate_order(x, n, k, out); }

void orc_trace(int on) {
    g_trace.on = on != 0;
    if (!on) g_trace.buf.clear();
}
int orc_trace_get(const char* name, float* out, int cap) {
    auto it = g_trace.buf.find(name);
    if (it == g_trace.buf.end()) return -1;
    int n = (int)it->second.size();
    if (out) std::memcpy(out, it->second.data(), sizeof(float) * std::min(n, cap));
    return n;
}

// Greedy decode as `needle bench --decode <steps>` drives the engine
// (crates/needle-cli/src/main.rs:566-587): prefill in chunks of 32 with
// LastLogits, then per step `next = argmax(logits)` and one decode forward of
// `next`. masks (optional, `steps` rows of ceil(vocab/8) bytes, bit set =
// allowed) apply the agent's ban (-1e30) before each argmax.
int orc_generate(void* mp, const uint32_t* prompt, int n, int steps, const uint8_t* masks, uint32_t* out_ids,
                 float* first_logits) {
    try {
        Model& m = *(Model*)mp;
        Session* s = session_new(m);
        std::vector<float> logits(m.c.out_rows());
        forward_native(m, *s, prompt, n, OUT_LAST_LOGITS, logits.data());
        if (first_logits) std::memcpy(first_logits, logits.data(), logits.size() * 4);
        size_t mb = (m.c.out_rows() + 7) / 8;
        for (int k = 0; k < steps; k++) {
            uint32_t next = masked_argmax(logits.data(), m.c.out_rows(), masks ? masks + k * mb : nullptr);
            out_ids[k] = next;
            forward_native(m, *s, &next, 1, OUT_LAST_LOGITS, logits.data());
        }
        delete s;
        return 0;
    } catch (std::exception& e) {
        g_err = e.what();
        return -1;
    }
}

// Many independent sequences on `threads` host threads (one sequence per
// thread at a time, dynamically assigned): the CPU baseline for the batched
// configs. prompts [S][n], masks [S][steps][mb] or null, out_ids [S][steps].
int orc_generate_batch(void* mp, int S, const uint32_t* prompts, int n, int steps, const uint8_t* masks, uint32_t* out_ids,
                       int threads) {
    Model& m = *(Model*)mp;
    size_t mb = (m.c.out_rows() + 7) / 8;
    std::atomic<int> next(0), bad(0);
    auto work = [&]() {
        t_no_team = true;  // a sequence a thread: no team inside
        for (;;) {
            int s = next.fetch_add(1);
            if (s >= S) return;
            if (orc_generate(mp, prompts + (size_t)s * n, n, steps, masks ? masks + (size_t)s * steps * mb : nullptr,
                             out_ids + (size_t)s * steps, nullptr) != 0)
                bad++;
        }
    };
    std::vector<std::thread> th;
    for (int k = 0; k < std::max(1, threads); k++) th.emplace_back(work);
    for (auto& t : th) t.join();
    return bad.load() ? -1 : 0;
}

// S sessions stepped together on host threads, for the timed CPU baseline of
// the batched decode config: prefill once, then each call is one greedy
// decode step of every session (masked argmax of its last logits, fed back).
struct OrcBatch {
    Model* m;
    std::vector<Session*> ss;
    std::vector<std::vector<float>> logits;
};

static void run_parallel(int S, int threads, const std::function<void(int)>& f) {
    std::atomic<int> next(0);
    auto work = [&]() {
        t_no_team = true;  // a sequence a thread: no team inside
        for (;;) {
            int s = next.fetch_add(1);
            if (s >= S) return;
            f(s);
        }
    };
    std::vector<std::thread> th;
    for (int k = 0; k < std::max(1, threads); k++) th.emplace_back(work);
    for (auto& t : th) t.join();
}

void* orc_batch_new(void* mp, int S) {
    OrcBatch* b = new OrcBatch();
    b->m = (Model*)mp;
    for (int s = 0; s < S; s++) b->ss.push_back(session_new(*b->m));
    b->logits.assign(S, std::vector<float>(b->m->c.out_rows()));
    return b;
}

void orc_batch_free(void* bp) {
    OrcBatch* b = (OrcBatch*)bp;
    for (auto s : b->ss) delete s;
    delete b;
}

int orc_batch_prefill(void* bp, const uint32_t* prompts, int n, int threads) {
    OrcBatch* b = (OrcBatch*)bp;
    std::atomic<int> bad(0);
    run_parallel((int)b->ss.size(), threads, [&](int s) {
        try {
            forward_native(*b->m, *b->ss[s], prompts + (size_t)s * n, n, OUT_LAST_LOGITS, b->logits[s].data());
        } catch (...) {
            bad++;
        }
    });
    return bad.load() ? -1 : 0;
}

int orc_batch_step(void* bp, const uint8_t* masks, uint32_t* next_ids, int threads) {
    OrcBatch* b = (OrcBatch*)bp;
    const int V = b->m->c.out_rows();
    const size_t mb = (V + 7) / 8;
    std::atomic<int> bad(0);
    run_parallel((int)b->ss.size(), threads, [&](int s) {
        try {
            uint32_t nx = masked_argmax(b->logits[s].data(), V, masks ? masks + s * mb : nullptr);
            if (next_ids) next_ids[s] = nx;
            forward_native(*b->m, *b->ss[s], &nx, 1, OUT_LAST_LOGITS, b->logits[s].data());
        } catch (...) {
            bad++;
        }
    });
    return bad.load() ? -1 : 0;
}

// Prefill-only throughput sample: S sequences of n tokens each, last-position
// logits per sequence into out [S][out_rows].
int orc_prefill_batch(void* mp, int S, const uint32_t* prompts, int n, float* out, int threads) {
    Model& m = *(Model*)mp;
    std::atomic<int> next(0), bad(0);
    auto work = [&]() {
        t_no_team = true;  // a sequence a thread: no team inside
        for (;;) {
            int s = next.fetch_add(1);
            if (s >= S) return;
            Session* ss = session_new(m);
            try {
                forward_native(m, *ss, prompts + (size_t)s * n, n, OUT_LAST_LOGITS, out ? out + (size_t)s * m.c.out_rows() : nullptr);
            } catch (...) {
                bad++;
            }
            delete ss;
        }
    };
    std::vector<std::thread> th;
    for (int k = 0; k < std::max(1, threads); k++) th.emplace_back(work);
    for (auto& t : th) t.join();
    return bad.load() ? -1 : 0;
}

// The synthetic archive (synth_archive) for the shape knobs: with out ==
// NULL only *len is set. 0 on success, -1 with orc_last_error.
int orc_synth_cact(int L, int vocab, int slots, int window, uint64_t global_mask, uint64_t site_mask, uint64_t seed,
                   float std_, const int* cq_bits, int n_cq_bits, unsigned heads, uint8_t* out, uint64_t cap,
                   uint64_t* len) {
    try {
        SynthSpec sp;
        sp.L = L;
        sp.vocab = vocab;
        sp.slots = slots;
        sp.window = window;
        sp.global_mask = global_mask;
        sp.site_mask = site_mask;
        sp.seed = seed;
        sp.std = std_;
        if (n_cq_bits > 0) sp.cq_bits.assign(cq_bits, cq_bits + n_cq_bits);
        sp.heads = heads;
        std::vector<uint8_t> b = synth_archive(sp);
        if (len) *len = b.size();
        if (out) {
            if (cap < b.size()) throw std::runtime_error("buffer too small");
            std::memcpy(out, b.data(), b.size());
        }
        return 0;
    } catch (std::exception& e) {
        g_err = e.what();
        return -1;
    }
}

// ---- the fused row ops alone (the fused-ops sweep's checker)

// infer.rs:426-443 (zcn) over rows x [T][n].
void orc_op_zcn(const float* x, const float* s, int T, int n, float* out) {
    for (int t = 0; t < T; t++) zcn(x + (size_t)t * n, s, out + (size_t)t * n, n);
}

// infer.rs:1716-1744 (chunk rows: sincosf of freq * pos) and the rotation of
// infer.rs:1474-1483 over 12 query heads then 2 key heads of 48, at
// positions 0 .. T-1; freq per infer.rs:938-946.
void orc_op_rope(const float* x, int T, float theta, float* out) {
    const int qk = 48, half = 24, heads = 14;
    if (T < 1) return;
    // the tables and a fresh session's chunk rows (direct angles)
    Model m;
    rope_tables(m, theta, qk);
    Session st;
    std::vector<float> cosv, sinv;
    rope_rows(m, st, 0, T, cosv, sinv);
    for (int t = 0; t < T; t++) {
        const float* cs = cosv.data() + (size_t)t * half;
        const float* sn = sinv.data() + (size_t)t * half;
        for (int h = 0; h < heads; h++) {
            const float* xi = x + (size_t)t * heads * qk + h * qk;
            float* o = out + (size_t)t * heads * qk + h * qk;
            for (int f = 0; f < half; f++) {
                const float a = xi[f], b = xi[f + half];
                o[f] = std::fmaf(-sn[f], b, cs[f] * a);
                o[f + half] = std::fmaf(sn[f], a, cs[f] * b);
            }
        }
    }
}

// infer.rs:2463-2496 (silu_native, scalar arm).
void orc_op_silu(const float* x, int64_t n, float* out) {
    std::memcpy(out, x, sizeof(float) * n);
    silu_div(out, x, n);
}

// qlinear.rs:309-323 (QMat::row) of the model's embedding for each id.
int orc_op_gather(void* mp, const uint32_t* ids, int T, float* out) {
    const Model& m = *(const Model*)mp;
    const int d = m.c.d;
    for (int t = 0; t < T; t++) {
        if ((int)ids[t] >= m.embedding.out) return -1;
        qmat_row(m.embedding, (int)ids[t], out + (size_t)t * d);
    }
    return 0;
}

}  // extern "C"
