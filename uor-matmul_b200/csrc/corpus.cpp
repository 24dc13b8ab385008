// corpus.cpp -- the reference's recorded xorshift fill, for tests and benchmarks.
#include <cstring>
#include "../../include/uor_b200_corpus.h"

extern "C" int uor_b200_corpus_fill(uint64_t salt, uint32_t kind, size_t count, void* out) {
    uint64_t s = 0x243F6A8885A308D3ull ^ salt;
    auto step = [&s]() {
        s ^= s << 13;
        s ^= s >> 7;
        s ^= s << 17;
        return s;
    };
    switch (kind) {
    case 0: {
        auto* o = static_cast<int8_t*>(out);
        for (size_t i = 0; i < count; ++i) o[i] = (int8_t)(step() >> 33);
        return 0;
    }
    case 1: {
        auto* o = static_cast<int32_t*>(out);
        for (size_t i = 0; i < count; ++i) o[i] = (int32_t)(uint32_t)step();
        return 0;
    }
    case 2: {
        auto* o = static_cast<uint64_t*>(out);
        for (size_t i = 0; i < count; ++i) o[i] = step() >> 33;
        return 0;
    }
    case 3: {
        auto* o = static_cast<uint8_t*>(out);
        std::memset(o, 0, (count + 1) / 2);
        for (size_t i = 0; i < count; ++i)
            o[i / 2] |= (uint8_t)(((step() >> 33) & 0xF) << (4 * (i % 2)));
        return 0;
    }
    case 4: {
        auto* o = static_cast<uint8_t*>(out);
        for (size_t i = 0; i < count; ++i) {
            const uint64_t v = step() >> 33;
            const bool masked = ((v >> 20) % 100) < 5;
            o[2 * i] = masked ? 0 : (uint8_t)(int8_t)((int)(v % 128) - 64);
            o[2 * i + 1] = masked ? 0 : 1;
        }
        return 0;
    }
    case 5: {
        auto* o = static_cast<uint32_t*>(out);
        for (size_t i = 0; i < count; ++i) {
            const uint64_t t = step();
            const uint32_t sign = (uint32_t)(t & 1);
            const uint32_t frac = (uint32_t)((t >> 33) & 0x7FFFFF);
            const int e = (int)((t >> 8) % 61) - 30;  // value exponent of the leading bit
            o[i] = (sign << 31) | ((uint32_t)(e + 127) << 23) | frac;
        }
        return 0;
    }
    default: return 7;
    }
}
