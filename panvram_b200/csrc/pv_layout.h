// pv_layout.h - the refrel3 v1 model constants (refrel3.h:24-66) and this build's device layout of a cohort:
// the per-assembly decode table that the window kernel reads, written on the host at open.
//
// Decode table (variable size per assembly, at most PV_TAB_MAX_BYTES). The reference keeps R3Tab {freq[61][104],
// cum[61][105], sym[61][4096]} = 275,354 B per assembly (refrel3.h:66); this layout answers the same question - which
// symbol s, with which frequency f and cumulative start, holds slot x & 4095 of context c - in typically 3-4 KB, so a
// cohort's tables stay L2-resident and each decoding warp can stage its assembly's table in shared memory:
//   cum8[61][8]     uint16  contexts with at most 6 symbols: cum[0..A], padded with cum[A]; the symbol is the number
//                           of cum[1..5] at or below the slot (a zero-frequency symbol is skipped by construction)
//   bidx[15][64]    uint8   contexts with 104 symbols: the index (in that context's dense list) of the symbol
//                           holding slot 64 k
//   doff[16]        uint16  the first dense entry of each 104-symbol context; doff[15] = entry count
//   dense[...]      uint32  each 104-symbol context's used symbols in order: cum | freq << 12 | sym << 25 (an unused
//                           context keeps one all-zero entry); a slot's symbol is found from bidx[slot >> 6] by
//                           stepping while slot >= cum + freq (at most 63 steps, typically 0-2)
// An all-zero context decodes as an error, as the reference's zero-frequency lookup does (refrel3.h:78).
#pragma once
#include <stdint.h>
#include "panvram_b200.h"

#if defined(__CUDACC__)
#define PV_HD __host__ __device__ __forceinline__
#else
#define PV_HD inline
#endif

namespace pvb {

enum { C_LL = 0, C_LITR = 4, C_LIT2 = 14, C_KIND = 31, C_DELTA = 47, C_REPK = 49, C_REPD = 50, C_DIR = 51, C_SELF = 52,
       C_LEN = 53, C_FLIPK = 59, C_FLIPD = 60, NCTX = 61 };
enum { K_CONT = 0, K_DELTA = 1, K_REP = 2, K_ABS = 3, K_SELF = 4, K_FLIP = 5 };
constexpr int AB = 104;
constexpr int NBIG = 15;
constexpr uint32_t PB = 12, MTOT = 1u << PB, RANS_L = 1u << 16, MINL = 12;

constexpr int TAB_CUM8 = 0;                        // uint16 [61][8]
constexpr int TAB_BUCKET = 64;                     // slots per bucket of the 104-symbol contexts' index
constexpr int TAB_BIDX = TAB_CUM8 + NCTX * 16;     // uint8 [15][64]
constexpr int TAB_DOFF = TAB_BIDX + NBIG * (4096 / TAB_BUCKET);   // uint16 [16]
constexpr int TAB_DENSE = TAB_DOFF + 16 * 2;       // uint32 [entries]
constexpr int TAB_MAX = TAB_DENSE + NBIG * AB * 4;
static_assert(TAB_MAX <= PV_TAB_MAX_BYTES, "decode table layout");
static_assert(TAB_DENSE % 4 == 0 && PV_TAB_MAX_BYTES % 16 == 0, "decode table alignment");

// symbols per context (refrel3.h:29-41)
PV_HD int alpha(int c) {
    if (c < C_LITR) return AB;
    if (c < C_DELTA) return 6;
    if (c < C_REPK) return AB;
    if (c == C_REPK) return 3;
    if (c == C_REPD) return AB;
    if (c == C_DIR) return 2;
    if (c == C_SELF) return AB;
    if (c < C_FLIPK) return AB;
    if (c == C_FLIPK) return 4;
    return AB;
}
// index of a 104-symbol context among the 15 of them, or -1
PV_HD int big_index(int c) {
    if (c < C_LITR) return c;                 // LL 0..3
    if (c < C_DELTA) return -1;
    if (c < C_REPK) return 4 + (c - C_DELTA); // DELTA 4..5
    if (c == C_REPD) return 6;
    if (c == C_SELF) return 7;
    if (c >= C_LEN && c < C_FLIPK) return 8 + (c - C_LEN);   // LEN 8..13
    if (c == C_FLIPD) return 14;
    return -1;
}
PV_HD uint32_t dense_entry(uint32_t cum, uint32_t freq, uint32_t sym) { return cum | (freq << 12) | (sym << 25); }
PV_HD uint32_t dense_cum(uint32_t e) { return e & 4095u; }
PV_HD uint32_t dense_freq(uint32_t e) { return (e >> 12) & 8191u; }
PV_HD uint32_t dense_sym(uint32_t e) { return e >> 25; }

// block table word 0: payload offset (40 bits) | payload length (24 bits); a length of PV_BLEN_BAD marks a block
// whose stream cannot be valid (longer than any refrel3 block stream can be) and decodes as an error
constexpr uint64_t PV_BLEN_BAD = (1ull << 24) - 1;
PV_HD uint64_t block_loc(uint64_t off, uint64_t len) { return off | ((len < PV_BLEN_BAD ? len : PV_BLEN_BAD) << 40); }
PV_HD uint64_t loc_off(uint64_t w) { return w & ((1ull << 40) - 1); }
PV_HD uint32_t loc_len(uint64_t w) { return (uint32_t)(w >> 40); }

}  // namespace pvb
