// state_file.h -- optimizer_states.bin layouts (host side).
//
// Version 2 is the reference's file (galore/src/state_file.rs:1-580), written
// and read byte for byte:
//   header, 64 bytes little-endian: magic "GALR" (0x47414C52), version,
//     num_layers, default rank, precision (0 = FP16 projectors, INT8 state),
//     header size (64), total size (u64), beta1, beta2, eps (f32),
//     step count (u64), 12 reserved bytes (state_file.rs:58-80);
//   one 20-byte descriptor per layer: m, n, rank (u32), byte offset (u64)
//     (:133-160);
//   per layer at its offset: P f16 m x r, Q f16 n x r, momentum i8 r x r,
//     variance i8 r x r, scale_m f32, scale_v f32 (:187-228).
// The f16 conversions are galore's own (project.rs:135-185): rounding adds
// half an ulp and truncates (halves round away from zero), the mantissa carry
// is ORed (not added) into the exponent, and NaN payloads keep only their top
// ten bits.
//
// Version 3 (no reference counterpart) holds the B200-mode state losslessly:
// the same header with version 3, 40-byte descriptors {m, n, rank, side,
// codec, block (u32), state elements (u64), byte offset (u64)}, and per layer
// the side's projector (bf16, s x r as stored), m8 and v8 (l x r), then the
// m and v block scales (f32, ceil(l r / block) each).
#pragma once
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include <vector>

namespace aeth {

constexpr uint32_t kStateMagic = 0x47414C52u;
constexpr uint32_t kStateHeaderSize = 64;
constexpr uint32_t kStateDescV2 = 20;
constexpr uint32_t kStateDescV3 = 40;

struct StateHeader {
    uint32_t magic = kStateMagic, version = 2, num_layers = 0, rank = 0, precision = 0,
             header_size = kStateHeaderSize;
    uint64_t total_size = 0;
    float beta1 = 0.9f, beta2 = 0.999f, eps = 1e-8f;
    uint64_t step_count = 0;
};

struct StateDesc {
    uint32_t m = 0, n = 0, rank = 0, side = 0, codec = 0, block = 0;
    uint64_t state_elems = 0, byte_offset = 0;
};

template <class T>
inline void put_le(std::vector<uint8_t>& b, size_t off, T v) {
    memcpy(b.data() + off, &v, sizeof(T));  // the supported hosts are little-endian
}
template <class T>
inline T get_le(const uint8_t* b) {
    T v;
    memcpy(&v, b, sizeof(T));
    return v;
}

inline void encode_state_header(const StateHeader& h, std::vector<uint8_t>& b) {
    put_le(b, 0, h.magic);
    put_le(b, 4, h.version);
    put_le(b, 8, h.num_layers);
    put_le(b, 12, h.rank);
    put_le(b, 16, h.precision);
    put_le(b, 20, h.header_size);
    put_le(b, 24, h.total_size);
    put_le(b, 32, h.beta1);
    put_le(b, 36, h.beta2);
    put_le(b, 40, h.eps);
    put_le(b, 44, h.step_count);
}

inline StateHeader decode_state_header(const uint8_t* b) {
    StateHeader h;
    h.magic = get_le<uint32_t>(b);
    h.version = get_le<uint32_t>(b + 4);
    h.num_layers = get_le<uint32_t>(b + 8);
    h.rank = get_le<uint32_t>(b + 12);
    h.precision = get_le<uint32_t>(b + 16);
    h.header_size = get_le<uint32_t>(b + 20);
    h.total_size = get_le<uint64_t>(b + 24);
    h.beta1 = get_le<float>(b + 32);
    h.beta2 = get_le<float>(b + 36);
    h.eps = get_le<float>(b + 40);
    h.step_count = get_le<uint64_t>(b + 44);
    return h;
}

// galore/src/project.rs:137-158 (f32 -> f16 bits).
inline uint16_t galore_f32_to_f16(float x) {
    uint32_t bits;
    memcpy(&bits, &x, 4);
    const uint16_t sign = (uint16_t)((bits >> 16) & 0x8000u);
    const int exp = (int)((bits >> 23) & 0xffu);
    const uint32_t frac = bits & 0x7fffffu;
    if (exp == 0xff) return (uint16_t)(sign | 0x7c00u | ((frac >> 13) & 0x3ffu));
    const int e = exp - 127 + 15;
    if (e >= 0x1f) return (uint16_t)(sign | 0x7c00u);
    if (e <= 0) {
        if (e < -10) return sign;
        const uint32_t mant = (frac | 0x800000u) >> (1 - e);
        return (uint16_t)(sign | ((mant + 0x1000u) >> 13));
    }
    return (uint16_t)(sign | ((uint32_t)e << 10) | ((frac + 0x1000u) >> 13));
}

// galore/src/project.rs:160-184 (f16 bits -> f32).
inline float galore_f16_to_f32(uint16_t h) {
    const uint32_t sign = h & 0x8000u, exp = (h >> 10) & 0x1fu;
    uint32_t frac = h & 0x3ffu, bits;
    if (exp == 0) {
        if (frac == 0) {
            bits = sign << 16;
        } else {
            uint32_t e = 0;
            while ((frac & 0x400u) == 0) { frac <<= 1; ++e; }
            frac &= 0x3ffu;
            bits = (sign << 16) | ((127 - 15 - e) << 23) | (frac << 13);
        }
    } else if (exp == 0x1f) {
        bits = (sign << 16) | 0x7f800000u | (frac << 13);
    } else {
        bits = (sign << 16) | ((exp + 127 - 15) << 23) | (frac << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

inline float bf16_bits_to_f32_host(uint16_t b) {
    const uint32_t u = (uint32_t)b << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

// Byte size of one layer section.
inline uint64_t state_section_v2(uint64_t m, uint64_t n, uint64_t r) { return 2 * m * r + 2 * n * r + 2 * r * r + 8; }
inline uint64_t state_section_v3(uint64_t s, uint64_t r, uint64_t elems, uint64_t blocks) {
    return 2 * s * r + 2 * elems + 8 * blocks;
}

}  // namespace aeth
