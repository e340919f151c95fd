// TEST INFRASTRUCTURE ONLY. This file is part of the CPU oracle: a C++ restatement of the
// reference CPU engine (crates/hardshell, crates/taco-coder). Only tests/, the smoke check
// and the CPU-baseline leg of bench.py may load it. The GPU product never links it.
//
// The integer rules of HardShell: rescale with round half up, clamp, floor division, the
// integer square root and the clamped table look-up. Each function follows one function of
// crates/hardshell/src/int.rs and gives the same value for every input.
#pragma once

#include <cstdint>
#include <cstddef>

namespace hso {

typedef __int128 i128;
typedef unsigned __int128 u128;

// int.rs:41 floor_div: the largest q with q*b <= a, for b > 0.
inline int64_t floor_div(int64_t a, int64_t b) {
    int64_t q = a / b;
    int64_t r = a % b;
    if (r != 0 && ((r < 0) != (b < 0))) q -= 1;
    return q;
}

// int.rs:110 shift_round: floor((p + 2^(s-1)) / 2^s), with an exact 0 for s > max_shift.
inline i128 shift_round(i128 p, uint32_t s, uint32_t max_shift) {
    if (s == 0) return p;
    if (s > max_shift) return 0;
    i128 half = (i128)1 << (s - 1);
    // The reference adds with wrapping arithmetic; the caller bounds keep it exact.
    u128 sum = (u128)p + (u128)half;
    return ((i128)sum) >> s;
}

// int.rs:63 rescale: floor((x*m + 2^(s-1)) / 2^s), product in i128, max shift 95.
inline i128 rescale(int64_t x, int32_t m, uint32_t s) {
    i128 product = (i128)x * (i128)m;
    return shift_round(product, s, 95);
}

// int.rs:85 rescale_wide: the same rule for an i128 input, wrapping product, max shift 126.
inline i128 rescale_wide(i128 x, int32_t m, uint32_t s) {
    u128 product = (u128)x * (u128)(i128)m;
    return shift_round((i128)product, s, 126);
}

// int.rs:102 rescale_wide_offset: floor((x*m + c + 2^(s-1)) / 2^s).
inline i128 rescale_wide_offset(i128 x, int32_t m, i128 c, uint32_t s) {
    u128 p = (u128)x * (u128)(i128)m + (u128)c;
    return shift_round((i128)p, s, 126);
}

// int.rs:131 clamp: max(lo, min(x, hi)); lo wins when the bounds cross.
inline int64_t clamp(int64_t x, int64_t lo, int64_t hi) {
    int64_t upper = x < hi ? x : hi;
    return upper > lo ? upper : lo;
}

// int.rs:138 clamp_wide.
inline int64_t clamp_wide(i128 x, int64_t lo, int64_t hi) {
    i128 upper = x < (i128)hi ? x : (i128)hi;
    i128 c = upper > (i128)lo ? upper : (i128)lo;
    return (int64_t)c;
}

inline int8_t clamp_act_i8(i128 x) { return (int8_t)clamp_wide(x, -127, 127); }
inline int16_t clamp_act_i16(i128 x) { return (int16_t)clamp_wide(x, -32767, 32767); }
inline int32_t clamp_i32(i128 x, int32_t lo, int32_t hi) { return (int32_t)clamp_wide(x, lo, hi); }

// int.rs:213 isqrt_u128: floor(sqrt(x)), digit by digit, two bits of x in each round.
inline u128 isqrt_u128(u128 x) {
    u128 bit = (u128)1 << 126;
    while (bit > x) bit >>= 2;
    u128 rem = x, res = 0;
    while (bit != 0) {
        u128 trial = res + bit;
        if (rem >= trial) {
            rem -= trial;
            res = (res >> 1) + bit;
        } else {
            res >>= 1;
        }
        bit >>= 2;
    }
    return res;
}

// int.rs:262 Table::lookup: the entry at clamp(index, 0, len - 1).
template <typename T>
inline T table_lookup(const T* entries, size_t len, int64_t index) {
    int64_t i = clamp(index, 0, (int64_t)len - 1);
    return entries[i];
}

}  // namespace hso
