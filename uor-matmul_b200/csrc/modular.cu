// modular.cu -- host planning of the modular route: the moduli prefix and the CRT constants.
#include "modular.cuh"

namespace uor {

namespace {

// 2^8, 3 5 17, 11 23, 13 19 and primes: pairwise coprime, largest first.
constexpr uint16_t kModuli[FM_MAX] = {256, 255, 253, 251, 247, 241, 239, 233, 229, 227,
                                      223, 211, 199, 197, 193, 191, 181, 179, 173, 167,
                                      163, 157, 151, 149, 139, 137, 131, 127, 113, 109,
                                      107, 103, 101, 97,  89,  83,  79,  73,  71,  67};

constexpr int HL = 14;  // 448-bit host integers
struct HBig {
    uint32_t l[HL];
};
void hb_set(HBig& x, uint32_t v) {
    for (auto& q : x.l) q = 0;
    x.l[0] = v;
}
void hb_mul(HBig& x, uint32_t v) {
    uint64_t c = 0;
    for (auto& q : x.l) {
        const uint64_t t = static_cast<uint64_t>(q) * v + c;
        q = static_cast<uint32_t>(t);
        c = t >> 32;
    }
}
uint32_t hb_div(HBig& x, uint32_t v) {  // x /= v, returns the remainder
    uint64_t r = 0;
    for (int i = HL - 1; i >= 0; --i) {
        const uint64_t cur = (r << 32) | x.l[i];
        x.l[i] = static_cast<uint32_t>(cur / v);
        r = cur % v;
    }
    return static_cast<uint32_t>(r);
}
void hb_ones(HBig& x, int bits) {  // x := 2^bits - 1
    for (auto& q : x.l) q = 0;
    for (int b = 0; b < bits; ++b) x.l[b >> 5] |= 1u << (b & 31);
}
void hb_mul_big(HBig& x, const HBig& y) {
    HBig r{};
    for (int i = 0; i < HL; ++i) {
        uint64_t c = 0;
        for (int j = 0; i + j < HL; ++j) {
            const uint64_t t = static_cast<uint64_t>(x.l[i]) * y.l[j] + r.l[i + j] + c;
            r.l[i + j] = static_cast<uint32_t>(t);
            c = t >> 32;
        }
    }
    x = r;
}
bool hb_less(const HBig& x, const HBig& y) {
    for (int i = HL - 1; i >= 0; --i)
        if (x.l[i] != y.l[i]) return x.l[i] < y.l[i];
    return false;
}
int hb_bits(const HBig& x) {
    for (int i = HL - 1; i >= 0; --i)
        if (x.l[i]) return 32 * i + 32 - __builtin_clz(x.l[i]);
    return 0;
}
uint32_t inv_mod(uint32_t a, uint32_t p) {
    int64_t t = 0, nt = 1, r = p, nr = a % p;
    while (nr) {
        const int64_t q = r / nr;
        const int64_t tt = t - q * nt;
        t = nt, nt = tt;
        const int64_t rr = r - q * nr;
        r = nr, nr = rr;
    }
    return static_cast<uint32_t>(t < 0 ? t + p : t);
}

}  // namespace

bool fm_plan_bound(const uint32_t* bound, int limbs, FmParams& f) {
    HBig need{};
    for (int i = 0; i < limbs && i < HL; ++i) need.l[i] = bound[i];
    if (hb_bits(need) > 32 * HL - 16) return false;
    hb_mul(need, (1u << 10) + 1);  // M 2^10 > (2^10 + 1) 2 bound
    hb_mul(need, 2);
    HBig M;
    hb_set(M, 1);
    int nm = 0;
    for (;; ++nm) {
        HBig scaled = M;
        hb_mul(scaled, 1u << 10);
        if (hb_less(need, scaled)) break;
        if (nm == FM_MAX) return false;
        hb_mul(M, kModuli[nm]);
    }
    if (nm == 0) hb_mul(M, kModuli[nm++]);
    if (nm & 1) {  // the kernels come in even moduli counts
        if (nm == FM_MAX) return false;
        hb_mul(M, kModuli[nm++]);
    }
    f = FmParams{};
    f.nm = nm;
    auto byte_of = [](const HBig& x, int b) {
        return static_cast<uint32_t>((x.l[b >> 2] >> (8 * (b & 3))) & 255u);
    };
    for (int l = 0; l < FM_MAX / 4 + 1; ++l) f.mm[l] = M.l[l];
    for (int b = 0; b < FM_MAX; ++b) f.nmb[b] = -static_cast<int32_t>(byte_of(M, b));
    for (int g = 0; g < nm; ++g) {
        const uint32_t p = kModuli[g];
        HBig mg = M;
        hb_div(mg, p);
        HBig t = mg;
        const uint32_t mgmod = hb_div(t, p);
        f.p[g] = p;
        f.inv[g] = inv_mod(mgmod, p);
        f.magic32[g] = static_cast<uint32_t>(((1ull << 32) + p - 1) / p);
        for (int b = 0; b < 4; ++b) f.mg[g / 4][b] |= ((f.magic32[g] >> (8 * b)) & 255u) << (8 * (g % 4));
        f.half[g] = p == 256 ? 127u : (p - 1) / 2;
        f.pneg[g] = 0u - p;
        f.hneg[g] = 0u - f.half[g];
        for (int b = 0; b < nm; ++b) f.md[g / 4][b] |= byte_of(mg, b) << (8 * (g % 4));
    }
    return true;
}

bool fm_plan_spans(int span_a, int span_b, size_t k, FmParams& f) {
    if (span_a <= 0 || span_b <= 0 || span_a + span_b > 300 || k > 0xFFFFFFFFull) return false;
    HBig b, y;
    hb_ones(b, span_a);
    hb_ones(y, span_b);
    hb_mul_big(b, y);
    hb_mul(b, static_cast<uint32_t>(k));
    return fm_plan_bound(b.l, HL, f);
}

bool fm_plan_ints(int bits, size_t k, FmParams& f) {
    if (bits <= 0 || bits > 64 || k > 0xFFFFFFFFull) return false;
    HBig b{};
    const int sh = 2 * bits - 2;
    b.l[sh >> 5] = 1u << (sh & 31);
    hb_mul(b, static_cast<uint32_t>(k));
    return fm_plan_bound(b.l, HL, f);
}

}  // namespace uor
