// pv_xxh3.h - XXH3_64bits (xxHash 0.8, seed 0, default secret) for inputs longer than 240 bytes, restated from its
// published algorithm in the pieces the device and the host split between them. The archive format names this hash
// for the source FASTA, the base stream and each block (FORMAT.md:11,26-27,51 of the reference), so its steps and
// constants must be XXH3's own.
//
// Eight 64-bit accumulators start at acc_init(i). The input is read in 1024-byte blocks of sixteen 64-byte stripes; for
// stripe s of a block and its little-endian word i (0..7), with d the word and k = d ^ secret word (s + i):
//     acc[i ^ 1] += d;   acc[i] += lo32(k) * hi32(k)
// After each of the (len - 1) / 1024 full blocks every accumulator is scrambled with secret word 16 + i:
//     acc ^= acc >> 47;  acc ^= key;  acc *= PRIME32_1
// Then the stripes of the last, partial block that lie wholly before byte len - 1 are accumulated the same way (no
// scramble), then the input's last 64 bytes with the secret from byte 121, and the result is
//     avalanche(len * PRIME64_1 + sum over pairs j < 4 of fold64((acc[2j] ^ s0) * (acc[2j + 1] ^ s1)))
// with s0, s1 the secret's words from byte 11 + 16 j, fold64 the xor of the 128-bit product's halves and
// avalanche(h) = h ^ h >> 37, * 0x165667919E3779F9, ^ >> 32.
// Within a block the updates only add, so a block's contribution is a sum that threads can form in any order and in
// parallel (pv_fasta.cu); only the scrambles between blocks form a serial chain.
// The 192-byte default secret is not written here: the host takes it at run time from the xxHash library's
// XXH3_generateSecret_fromSeed with seed 0, which returns the default secret itself.
#pragma once
#include <stdint.h>
#include <string.h>

#if defined(__CUDACC__)
#define PV_XH __host__ __device__ __forceinline__
#else
#define PV_XH inline
#endif

namespace pvx {

constexpr uint64_t PRIME32_1 = 0x9E3779B1ull, PRIME32_2 = 0x85EBCA77ull, PRIME32_3 = 0xC2B2AE3Dull;
constexpr uint64_t PRIME64_1 = 0x9E3779B185EBCA87ull, PRIME64_2 = 0xC2B2AE3D27D4EB4Full, PRIME64_3 = 0x165667B19E3779F9ull,
                   PRIME64_4 = 0x85EBCA77C2B2AE63ull, PRIME64_5 = 0x27D4EB2F165667C5ull;
constexpr uint64_t AVALANCHE = 0x165667919E3779F9ull;
constexpr int SECRET_BYTES = 192, STRIPE = 64, BLOCK = 1024, STRIPES_PER_BLOCK = 16;
constexpr int SCRAMBLE_AT = SECRET_BYTES - STRIPE;            // secret byte of the scramble keys (128)
constexpr int LAST_STRIPE_AT = SECRET_BYTES - STRIPE - 7;     // secret byte of the last stripe's keys (121)
constexpr int MERGE_AT = 11;                                  // secret byte of the merge keys
constexpr uint64_t LONG_INPUT = 241;                          // the long-input path applies from this length

PV_XH uint64_t acc_init(int i) {
    return i == 0 ? PRIME32_3 : i == 1 ? PRIME64_1 : i == 2 ? PRIME64_2 : i == 3 ? PRIME64_3
         : i == 4 ? PRIME64_4 : i == 5 ? PRIME32_2 : i == 6 ? PRIME64_5 : PRIME32_1;
}
PV_XH uint64_t rd64(const uint8_t* p) { uint64_t v; memcpy(&v, p, 8); return v; }   // little-endian hosts and GPUs
PV_XH uint64_t mul32x32(uint64_t k) { return (k & 0xFFFFFFFFull) * (k >> 32); }
PV_XH uint64_t scramble(uint64_t a, uint64_t key) { a ^= a >> 47; a ^= key; return a * PRIME32_1; }
PV_XH uint64_t avalanche(uint64_t h) { h ^= h >> 37; h *= AVALANCHE; return h ^ (h >> 32); }

// the 8-word keys the device needs, taken out of the secret once (all offsets the device uses are multiples of 8
// except the last stripe's and the merge's, which get their own arrays)
struct Keys {
    uint64_t w[24];        // secret words 0..23 (stripe keys: word s + i; scramble keys: words 16..23)
    uint64_t last[8];      // the last stripe's keys (secret bytes 121 + 8 i)
    uint64_t merge[8];     // the merge keys (secret bytes 11 + 8 i)
};
inline void keys_from_secret(const uint8_t* secret, Keys* k) {
    for (int i = 0; i < 24; i++) k->w[i] = rd64(secret + 8 * i);
    for (int i = 0; i < 8; i++) k->last[i] = rd64(secret + LAST_STRIPE_AT + 8 * i);
    for (int i = 0; i < 8; i++) k->merge[i] = rd64(secret + MERGE_AT + 8 * i);
}
// one stripe into acc (host; the device spreads a block's stripes over a warp)
PV_XH void stripe(uint64_t acc[8], const uint8_t* in, const uint64_t* key8) {
    for (int i = 0; i < 8; i++) {
        const uint64_t d = rd64(in + 8 * i);
        acc[i ^ 1] += d;
        acc[i] += mul32x32(d ^ key8[i]);
    }
}
PV_XH uint64_t fold64(uint64_t a, uint64_t b) {
#if defined(__CUDA_ARCH__)
    return (a * b) ^ __umul64hi(a, b);
#else
    const unsigned __int128 p = (unsigned __int128)a * b;
    return (uint64_t)p ^ (uint64_t)(p >> 64);
#endif
}
PV_XH uint64_t merge(const uint64_t acc[8], const uint64_t* mkey, uint64_t len) {
    uint64_t r = len * PRIME64_1;
    for (int j = 0; j < 4; j++) r += fold64(acc[2 * j] ^ mkey[2 * j], acc[2 * j + 1] ^ mkey[2 * j + 1]);
    return avalanche(r);
}

}  // namespace pvx
