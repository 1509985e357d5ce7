// pv_kernels.cu - the refrel3 v1 window decode on sm_100a (pv_windows of include/panvram_b200.h).
//
// Replaces the reference's three-kernel path (pv_queue_kernel -> pv_case_kernel -> pv_rc_tok_kernel,
// pv_cuda.cu:38-147) with kernels that write every output byte once. Work item = (window, one stride cell of a block
// it touches): with the cohort's checkpoint index (built at open by pv_index_kernel, which decodes every block once)
// an item decodes from the checkpoint at or before its cell to the end of its output range; without an index the
// cell is the whole block.
//
// The fused form, pv_windows_kernel (calls of few items: split_min_items), one item per warp, WARPS warps per CTA:
//   * lane 0 stages into the warp's shared slot, with TMA bulk copies completing on one mbarrier (bounded wait:
//     status 4), the assembly's compact decode table (pv_layout.h), the item's rANS stream and the reference span
//     its diagonal covers; then it decodes (every validity check of refrel3.h:114-160 on a block's full decode, so a
//     corrupt block reports status 1 exactly as the reference does) with the decoder state in registers, keeping
//     only the ops and literal bytes that land inside the item's range.
//   * the warp then writes the item's output range in 16-byte vector stores (emit_ops): chunks inside one op first
//     (lane i every 32nd chunk; reference copies realigned with funnel shifts, literals from the item's array), then
//     the chunks around op boundaries, one lane each; lower-case runs, reverse complement and the token map (or the
//     fused token-id map) are applied in registers before each store.
//   * items from the cohort's block cache (decoded once at open) are copied from it.
//   * items needing the general path (a self copy inside the window, or more ops / literals than a slot holds) are
//     decoded again by the whole CTA into a Q-byte block buffer in the caller's scratch, ops executed in order, then
//     emitted the same way.
// The split form (larger calls): pv_decode_kernel decodes one item per lane (as many per warp as keep about 3,072
// decode warps in flight; tables through L1; the item's reference span warmed into L2) into a plan in the caller's
// scratch, with the item's lower-case runs; pv_emit_kernel, persistent, emits one item per warp from a queue, reading
// the plan in place (reverse-complement copies read forward from the reverse-complemented reference); pv_heavy_kernel
// takes the general-path items.
// Also here: pv_sample_coords_kernel, sample()'s coordinate arithmetic and (pv_sample_draw_coords) the draws torch's
// randint / rand would make, restated on curand's Philox states; small kernels that move window coordinates from and
// the status word to pinned host memory without a copy engine. The window kernels are launched with programmatic
// dependent launch and wait for their predecessor in griddepcontrol.wait.
#include <cuda_runtime.h>
#include <curand_kernel.h>
#include <stdint.h>
#include <stdio.h>

#include <algorithm>
#include <atomic>
#include <utility>
#include <type_traits>

#include "pv_layout.h"

namespace {

using namespace pvb;

constexpr int CTA = 128;
constexpr int OPS_CAP = 64;    // ops inside the window per item (common path)
constexpr int LIT_CAP = 128;   // literal bytes inside the window per item
constexpr int RUN_CAP = 8;     // lower-case runs per item kept in shared memory
constexpr int HOPS = 64;       // ops per chunk on the heavy path

enum { ST_IDLE = 0, ST_OK = 1, ST_HEAVY = 2, ST_ERR = 3, ST_CACHED = 4, ST_LOCATED = 5 };
enum { DEC_DONE = 1, DEC_PAUSE = 0, DEC_ERR = -1, DEC_ABORT = -2 };

struct Op { uint32_t src; uint16_t dk; uint16_t len; };   // dk: block offset | kind << 14 (8 bytes: src, then dk | len << 16)
static_assert(sizeof(Op) == 8, "Op is read as two words");
__device__ __forceinline__ uint32_t op_dst(const Op& o) { return o.dk & 0x3FFFu; }
__device__ __forceinline__ uint32_t op_kind(const Op& o) { return o.dk >> 14; }

struct __align__(16) Item {
    int64_t w;              // window index
    uint64_t s;             // window start in the assembly's stream
    uint64_t bst;           // block start in the stream
    uint64_t gblk;          // pooled block index
    const uint8_t* cptr;    // the block's decoded bytes in the cohort's block cache (ST_CACHED)
    uint64_t poff;          // its stream: offset in the pooled payload
    int64_t pst;            // its start state c << 1 | dir
    uint64_t grp;           // compact block table: its group, its index in the group, the group's block count
    uint32_t gj, gm;
    uint32_t plen;          // its stream's length
    uint32_t staged;        // the stream was copied into the slot
    uint64_t tab_off;       // the assembly's decode table in the pooled tables
    int32_t a;              // assembly
    uint32_t ox0, ox1, blen;
    int32_t state;
    uint16_t nops, nlits;
    uint32_t run_first, run_cnt;
    uint32_t tab_bytes, span_len;   // span_len: bytes of the reference staged in the slot (from position span_lo)
    int64_t span_lo;
    uint64_t ck;            // its decode's starting checkpoint in the cohort's index, or NO_CK (the block's start)
    uint64_t cpos;          // that checkpoint's stream position in the pooled payload
    int64_t cst;            // the current diagonal c << 1 | dir where the decode starts (the spans follow it)
    uint32_t co;            // the block offset where the decode starts
    uint32_t jc, wx0, wx1;  // its cell of the block; the window's bytes in the block [wx0, wx1)
    uint4 landing;          // 16 bytes a bulk copy may target (the expired-wait test's completing copy)
    uint64_t idx;           // its index in the call (the trace record it writes)
    alignas(16) int32_t runs[2 * RUN_CAP];   // window-relative [start, end), clipped to the item's range
    alignas(16) Op ops[OPS_CAP];
    alignas(16) uint8_t lits[LIT_CAP];
};
// an Item is copied in 16-byte words: the part up to its ops (header and runs), then only the ops and literal bytes it
// holds
constexpr uint32_t ITEM_HEAD16 = (uint32_t)(offsetof(Item, ops) / 16), ITEM_LITS16 = (uint32_t)(offsetof(Item, lits) / 16);
static_assert(offsetof(Item, ops) % 16 == 0 && offsetof(Item, lits) % 16 == 0 && sizeof(Item) % 16 == 0, "Item layout");

struct Params {
    pv_dev_cohort C;
    const int64_t* wasm; const int64_t* wstart; const uint8_t* rc;
    uint8_t* out; int32_t* status; uint8_t* wstatus;
    uint8_t* work;                 // block-path buffers in global memory: Q bytes per CTA
    uint64_t n, W, bpw, total;
    uint32_t slot_bytes, tab_area, pay_cap, span_cap;   // a warp's shared slot: Item | table | payload | reference span
    int tokens, apply_case, force_block;
    int test_wait;                 // PV_WIN_TEST_WAIT: every slot's barrier expects 16 bytes more than its copies bring
    uint32_t qshift;               // log2 of the block size
    int narrow;                    // windows shorter than a block: stage only the span under the output range
    int64_t* out64;                // token-id output (pv_windows_ids): int64 [n, W]; then `out` is unused
    int64_t ids[5];                // the ids of tokens 0..4
    uint32_t dec_lanes;            // split form: items per decode warp (one per lane, lanes 0 .. dec_lanes - 1)
    uint32_t cshift;               // log2 of an item's cell: the checkpoint stride, or the block size without an index
    uint64_t* trace;               // pv_windows_trace: 8 words per item, or NULL
};
constexpr uint64_t NO_CK = ~0ull;

// The trace (pv_windows_trace): per item, %globaltimer (ns) when it reaches each phase - 0 start, 1 located (block,
// checkpoint, case runs), 2 its decode starts (the fused kernel: its slot's copies have landed), 3 decoded, 4 the
// emission kernel takes it (split form), 5 its header is in the emission warp's slot, 6 emitted - and word 7: SM |
// state << 8 | form << 12 (1 fused, 2 split) | from a checkpoint << 14 | ops << 16 | literals << 32 | decoded bases << 48.
__device__ __forceinline__ uint64_t gtime() { uint64_t t; asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t)); return t; }
__device__ __forceinline__ void trace_at(const Params& P, uint64_t item, int k) { if (P.trace) P.trace[item * 8 + k] = gtime(); }
template <class It>
__device__ __forceinline__ void trace_done(const Params& P, const It* it, int form) {
    if (!P.trace) return;
    uint32_t sm;
    asm volatile("mov.u32 %0, %%smid;" : "=r"(sm));
    P.trace[it->idx * 8 + 6] = gtime();
    const uint64_t dec = it->ox1 > it->co ? it->ox1 - it->co : 0;
    P.trace[it->idx * 8 + 7] = (uint64_t)(sm & 0xFF) | ((uint64_t)(it->state & 15) << 8) | ((uint64_t)form << 12) |
                               ((uint64_t)(it->ck != ~0ull) << 14) | ((uint64_t)it->nops << 16) | ((uint64_t)it->nlits << 32) | (dec << 48);
}

// status bits into the call's word and, when asked, into the window's byte (4-byte aligned, padded array)
__device__ __forceinline__ void report(const Params& P, uint64_t w, int bits) {
    atomicOr(P.status, bits);
    if (P.wstatus) atomicOr((unsigned int*)(P.wstatus + (w & ~3ull)), (unsigned int)bits << (8 * (w & 3)));
}

// shared-memory loads by 32-bit shared address (the decode tables are staged there by a TMA bulk copy)
__device__ __forceinline__ uint4 lds128(uint32_t a) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
    return v;
}
__device__ __forceinline__ uint32_t lds32(uint32_t a) { uint32_t v; asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a)); return v; }
__device__ __forceinline__ uint32_t lds16(uint32_t a) { uint16_t v; asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(a)); return v; }
__device__ __forceinline__ uint32_t lds8(uint32_t a) { uint16_t v; asm volatile("ld.shared.u8 %0, [%1];" : "=h"(v) : "r"(a)); return v; }
__device__ __forceinline__ uint32_t smem_addr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ uint32_t cum_at(uint4 r, uint32_t k) {
    const uint32_t w = (k >> 1) == 0 ? r.x : (k >> 1) == 1 ? r.y : (k >> 1) == 2 ? r.z : r.w;
    return (k & 1) ? (w >> 16) : (w & 0xFFFFu);
}
// ---------------------------------------------------------------- rANS decoder (refrel3.h:69-109)
// The block's rANS stream: staged in shared memory (32-bit shared addresses) or read from global memory. peek(k) is
// the byte k ahead, or anything when that is past the end (the caller checks left() before using it): the shared
// variant may read the next bytes of the warp's slot, the global one reads nothing past the end.
struct SmemStream {
    uint32_t p, e;
    __device__ __forceinline__ uint32_t peek(uint32_t k) const { return lds8(p + k); }
    __device__ __forceinline__ uint32_t left() const { return e - p; }
    __device__ __forceinline__ void skip(uint32_t k) { p += k; }
};
struct GlobalStream {
    const uint8_t* p; const uint8_t* e;
    __device__ __forceinline__ uint32_t peek(uint32_t k) const { return p + k < e ? (uint32_t)__ldg(p + k) : 0u; }
    __device__ __forceinline__ uint32_t left() const { return (uint32_t)(e - p); }
    __device__ __forceinline__ void skip(uint32_t k) { p += k; }
};
// a validated block's stream read from a checkpoint: no end to check (the decode to the item's end reads no further
// than the block's stream, plus the two bytes a step looks ahead, inside the pool's padding)
struct OpenStream {
    const uint8_t* p;
    __device__ __forceinline__ uint32_t peek(uint32_t k) const { return (uint32_t)__ldg(p + k); }
    __device__ __forceinline__ uint32_t left() const { return 1u << 30; }
    __device__ __forceinline__ void skip(uint32_t k) { p += k; }
};
// The decoder state is all scalar - the four-entry diagonal cache as named registers, indexed by selects - so that,
// inlined, the block's serial rANS chain stays in registers and never round-trips through local memory.
template <class S>
struct Dec {
    S st;
    uint32_t x; int bad;
    uint32_t o, li, pk; int nc;                          // pk: previous kind + 1 (0: none yet)
    uint64_t c0, c1, c2, c3; uint32_t d0, d1, d2, d3;   // diagonal cache, most recent first
};

// byte renormalisation (refrel3.h:80,87). A step leaves x >= 16, so a well-formed stream needs at most two bytes:
// both are loaded before x is known (their latency overlaps the symbol's table lookup) and taken branch-free. Running
// out of stream sets `bad` (sticky); the decoder then carries on with whatever state it has until the event's next
// check, exactly where the reference's check catches it (refrel3.h:125,147), so the outcome - a failed block - is the
// same. A state still below 2^16 after two bytes (only a corrupt stream, e.g. a zero initial state) continues byte by
// byte as the reference does.
struct SlowRenorm { uint32_t x, used; int bad; };
template <class S>
__device__ __noinline__ SlowRenorm renorm_slow(uint32_t x, S st) {   // by value: the decoder state stays in registers
    SlowRenorm r{x, 0, 0};
    while (r.x < RANS_L) {
        if (st.left() == 0) { r.bad = 1; break; }
        r.x = (r.x << 8) | st.peek(0);
        st.skip(1);
        r.used++;
    }
    return r;
}
template <class S>
__device__ __forceinline__ void renorm(Dec<S>& d, uint32_t b0, uint32_t b1) {
    uint32_t x = d.x;
    const uint32_t left = d.st.left();
    const uint32_t r1 = x < RANS_L;
    x = r1 ? (x << 8) | b0 : x;
    const uint32_t r2 = x < RANS_L;
    x = r2 ? (x << 8) | b1 : x;
    const uint32_t used = r1 + r2;
    d.bad |= (int)(used > left);
    d.st.skip(used > left ? left : used);
    d.x = x;
    if (x < RANS_L) {
        const SlowRenorm r = renorm_slow(x, d.st);
        d.x = r.x; d.st.skip(r.used); d.bad |= r.bad;
    }
}
// one rANS step: a zero-frequency lookup (refrel3.h:78) sets bad
template <class S>
__device__ __forceinline__ uint32_t rans_step(Dec<S>& d, uint32_t slot, uint32_t s, uint32_t f, uint32_t cm, uint32_t b0, uint32_t b1) {
    d.bad |= (int)(f == 0);
    d.x = f * (d.x >> PB) + slot - cm;
    renorm(d, b0, b1);
    return s;
}
// An assembly's decode table (pv_layout.h), staged in shared memory (32-bit shared address) or read in place from
// global memory through the L1 cache.
struct SmemTab {
    uint32_t b;
    __device__ __forceinline__ uint4 row(int c) const { return lds128(b + TAB_CUM8 + c * 16); }
    __device__ __forceinline__ uint32_t doff(int bi) const { return lds16(b + TAB_DOFF + 2 * bi); }
    __device__ __forceinline__ uint32_t bidx(int bi, uint32_t k) const { return lds8(b + TAB_BIDX + bi * (4096 / TAB_BUCKET) + k); }
    __device__ __forceinline__ uint32_t dense(uint32_t u) const { return lds32(b + TAB_DENSE + 4 * u); }
};
struct GlobalTab {
    const uint8_t* b;
    __device__ __forceinline__ uint4 row(int c) const { return __ldg((const uint4*)(b + TAB_CUM8 + c * 16)); }
    __device__ __forceinline__ uint32_t doff(int bi) const { return __ldg((const uint16_t*)(b + TAB_DOFF) + bi); }
    __device__ __forceinline__ uint32_t bidx(int bi, uint32_t k) const { return __ldg(b + TAB_BIDX + bi * (4096 / TAB_BUCKET) + k); }
    __device__ __forceinline__ uint32_t dense(uint32_t u) const { return __ldg((const uint32_t*)(b + TAB_DENSE) + u); }
};
// one symbol of a context with at most 6 symbols: the table's cum8 row
template <class S, class Tb>
__device__ __forceinline__ uint32_t dsym_small(Dec<S>& d, const Tb& T, int c) {
    const uint32_t b0 = d.st.peek(0), b1 = d.st.peek(1);
    const uint32_t slot = d.x & (MTOT - 1);
    const uint4 r = T.row(c);
    const uint32_t s = (uint32_t)((r.x >> 16) <= slot) + (uint32_t)((r.y & 0xFFFFu) <= slot) + (uint32_t)((r.y >> 16) <= slot) +
                       (uint32_t)((r.z & 0xFFFFu) <= slot) + (uint32_t)((r.z >> 16) <= slot);
    const uint32_t cm = cum_at(r, s);
    return rans_step(d, slot, s, cum_at(r, s + 1) - cm, cm, b0, b1);
}
// one symbol of a 104-symbol context, bi its index among the 15 of them (pv_layout.h big_index)
template <class S, class Tb>
__device__ __forceinline__ uint32_t dsym_big(Dec<S>& d, const Tb& T, int bi) {
    const uint32_t b0 = d.st.peek(0), b1 = d.st.peek(1);
    const uint32_t slot = d.x & (MTOT - 1);
    uint32_t u = T.doff(bi) + T.bidx(bi, slot / TAB_BUCKET);
    uint32_t e = T.dense(u);
    while (dense_freq(e) && slot >= dense_cum(e) + dense_freq(e)) e = T.dense(++u);
    return rans_step(d, slot, dense_sym(e), dense_freq(e), dense_cum(e), b0, b1);
}
// raw bits (at most 32), at most 16 per step (refrel3.h:83-90)
template <class S>
__device__ __forceinline__ uint32_t draw(Dec<S>& d, uint32_t nb) {
    uint32_t v = 0, sh = 0;
    while (nb) {
        const uint32_t b0 = d.st.peek(0), b1 = d.st.peek(1);
        const uint32_t k = nb > 16 ? 16 : nb;
        const uint32_t b = d.x & ((1u << k) - 1);
        d.x >>= k;
        renorm(d, b0, b1);
        v |= b << sh; sh += k; nb -= k;
    }
    return v;
}
// bucketed value (refrel3.h:91): 16 small buckets, then 4 per octave with (s - 16) / 4 + 2 raw bits; s < 104 keeps it
// below 2^26
__device__ __forceinline__ uint32_t unbucket(uint32_t s, uint32_t extra) {
    if (s < 16) return s;
    const uint32_t e = (s - 16) / 4 + 4, m = (s - 16) & 3;
    return (1u << e) | (m << (e - 2)) | extra;
}
template <class S, class Tb>
__device__ __forceinline__ uint32_t dval_big(Dec<S>& d, const Tb& T, int bi) {
    const uint32_t s = dsym_big(d, T, bi);
    return unbucket(s, draw(d, s < 16 ? 0 : (s - 16) / 4 + 2));
}
// class of the previous kind (none 0, CONT 1, DELTA / REP / FLIP 2, ABS / SELF 3) from pk = previous kind + 1
__device__ __forceinline__ uint32_t kclass(uint32_t pk) { return (0x2332210u >> (4 * pk)) & 3u; }
__device__ __forceinline__ uint32_t llc(uint32_t ll) { return (uint32_t)(ll > 0) + (uint32_t)(ll > 1) + (uint32_t)(ll > 8); }
__device__ __forceinline__ int32_t unzz(uint32_t z) { return (int32_t)(z >> 1) ^ -(int32_t)(z & 1); }
__device__ __forceinline__ uint8_t comp_up(uint8_t c) { return c == 'A' ? 'T' : c == 'C' ? 'G' : c == 'G' ? 'C' : c == 'T' ? 'A' : c; }
// The reference as a block reads it: the span its start diagonal covers, staged in shared memory by the item's TMA
// copy, and global memory (64 readable bytes on each side of the reference) for any position off that span.
// With the packed reference (pw != NULL) the off-span reads unpack 2-bit words and look the position up in the runs of
// other bytes (bucket index, then a short forward scan that the sentinel run ends).
struct RefView {
    const uint8_t* g; uint64_t n;           // global reference (byte form) and its length
    int64_t lo; uint32_t len; uint32_t sm;  // staged span: reference positions [lo, lo + len) at shared address sm
    const uint32_t* pw; const pv_ref_run* runs; const uint32_t* pidx;   // packed form, or pw == NULL
    __device__ __forceinline__ uint32_t packed_byte(int64_t q) const {   // 0 <= q < n
        uint32_t b = (0x54474341u >> (8 * ((__ldg(pw + (q >> 4)) >> ((q & 15) * 2)) & 3u))) & 0xFFu;
        for (uint32_t i = __ldg(pidx + (q >> PV_REF_BUCKET_SHIFT));; i++) {
            const uint64_t rs = __ldg(&runs[i].start);
            const uint32_t rl = __ldg(&runs[i].len);
            if (rs + rl > (uint64_t)q) { if (rs <= (uint64_t)q) b = __ldg(&runs[i].byte); break; }
        }
        return b;
    }
    __device__ __forceinline__ uint32_t byte(int64_t q) const {        // 0 <= q < n
        if ((uint64_t)(q - lo) < (uint64_t)len) return lds8(sm + (uint32_t)(q - lo));
        return pw ? packed_byte(q) : (uint32_t)__ldg(g + q);
    }
};
// the reference base the diagonal predicts at block offset o: 0..3, 4 = none (refrel3.h:104-109); refcode maps the
// reference byte b at that position
__device__ __forceinline__ int refcode(uint32_t b, uint32_t dir) {
    const uint32_t k = ((b >> 1) ^ (b >> 2)) & 3u;                 // A 0, C 1, G 2, T 3 for those letters
    if (((0x54474341u >> (8 * k)) & 0xFFu) != b) return 4;         // not an upper-case A, C, G or T
    return (int)(dir ? k ^ 3u : k);                                // the complement's code on the reverse strand
}
__device__ __forceinline__ int refbase(const RefView& R, uint64_t c, uint32_t dir, uint32_t o) {
    const int64_t q = dir ? (int64_t)c - (int64_t)o : (int64_t)c + (int64_t)o;
    if (q < 0 || (uint64_t)q >= R.n) return 4;
    return refcode(R.byte(q), dir);
}
template <class S>
__device__ __forceinline__ void dget(const Dec<S>& d, int k, uint64_t& c, uint32_t& dir) {
    c = k == 0 ? d.c0 : k == 1 ? d.c1 : k == 2 ? d.c2 : d.c3;
    dir = k == 0 ? d.d0 : k == 1 ? d.d1 : k == 2 ? d.d2 : d.d3;
}
// move-to-front push of a diagonal (refrel3.h:98-102)
template <class S>
__device__ __forceinline__ void dpush(Dec<S>& d, uint64_t c, uint32_t dir) {
    int j = (d.nc > 0 && d.c0 == c && d.d0 == dir) ? 0 : (d.nc > 1 && d.c1 == c && d.d1 == dir) ? 1
          : (d.nc > 2 && d.c2 == c && d.d2 == dir) ? 2 : (d.nc > 3 && d.c3 == c && d.d3 == dir) ? 3 : -1;
    if (j < 0) { if (d.nc < 4) d.nc++; j = d.nc - 1; }
    if (j >= 3) { d.c3 = d.c2; d.d3 = d.d2; }
    if (j >= 2) { d.c2 = d.c1; d.d2 = d.d1; }
    if (j >= 1) { d.c1 = d.c0; d.d1 = d.d0; }
    d.c0 = c; d.d0 = dir;
}
template <class S>
__device__ __forceinline__ void dec_init(Dec<S>& d, const S& src, int64_t st) {
    d.st = src; d.bad = 0; d.x = 0;
    d.o = 0; d.li = 0; d.pk = 0; d.nc = 1;
    d.c0 = (uint64_t)(st >> 1); d.d0 = (uint32_t)(st & 1);
    d.c1 = d.c2 = d.c3 = 0; d.d1 = d.d2 = d.d3 = 0;
    if (d.st.left() < 3) { d.bad = 1; return; }
    d.x = d.st.peek(0) | (d.st.peek(1) << 8) | (d.st.peek(2) << 16);
    d.st.skip(3);
}

// The decoder at a checkpoint of the cohort's index (include/panvram_b200.h pv_ckpt): src reads the block's stream from
// the byte the checkpoint had reached (ck_pos).
__device__ __forceinline__ uint64_t ck_diag(uint32_t lo, uint32_t hi) { return (((uint64_t)(hi & 0x7Fu) << 32) | lo) - (uint64_t)PV_CKPT_BIAS; }
// a checkpoint's stream position in the pooled payload: p, and bits 32..39 in its flags' high byte
__device__ __forceinline__ uint64_t ck_pos(uint32_t p, uint32_t ow) { return ((uint64_t)(ow >> 24) << 32) | p; }
template <class S>
__device__ __forceinline__ void dec_init_ck(Dec<S>& d, const S& src, const pv_ckpt* ck) {
    const uint4 a = __ldg((const uint4*)ck), b = __ldg((const uint4*)ck + 1);
    d.st = src; d.bad = 0;
    d.x = a.x & 0xFFFFFFu; d.pk = (a.x >> 24) & 7u; d.nc = (int)((a.x >> 27) & 3u) + 1;
    d.o = b.w & 0xFFFFu; d.li = 0;
    d.c0 = ck_diag(a.z, b.z); d.c1 = ck_diag(a.w, b.z >> 8); d.c2 = ck_diag(b.x, b.z >> 16); d.c3 = ck_diag(b.y, b.z >> 24);
    d.d0 = (b.z >> 7) & 1u; d.d1 = (b.z >> 15) & 1u; d.d2 = (b.z >> 23) & 1u; d.d3 = b.z >> 31;
}

// The event loop of refrel3.h:114-160, from the decoder's state (a block's start or a checkpoint) until the output
// reaches `stop`. From a block's start with stop = blen it is the whole block, with the end-of-stream checks of
// refrel3.h:157; from a checkpoint (validated: the cohort's index decoded the block in full at open) it is an item's
// range, ending with the event that reaches `stop`, and the end-of-stream checks are not repeated (the stream's end
// may not be known: a decode from a checkpoint can read the pooled payload with no end but its padding). Sinks: at(d)
// sees the state at each event boundary, more() is asked before each event (false pauses, resumable), lit()/op()
// returning false abort the decode (the caller takes another path). Returns DEC_*.
template <class S, class Sink, class Tb>
__device__ __forceinline__ int decode_events(Dec<S>& d, const Tb& T, const RefView& R, uint32_t blen, uint32_t stop, Sink& sk,
                                             bool validated = false) {
    const uint64_t ref_n = R.n;
    if (d.bad) return DEC_ERR;
    while (d.o < stop) {
        sk.at(d);
        if (!sk.more()) return DEC_PAUSE;
        // the reference byte a first literal's context reads (refbase at d.o), loaded before the LL symbol is decoded
        // so that its latency overlaps the symbol's table lookups (the byte form; the packed form looks it up after)
        const int64_t q0 = d.d0 ? (int64_t)d.c0 - (int64_t)d.o : (int64_t)d.c0 + (int64_t)d.o;
        const bool in0 = q0 >= 0 && (uint64_t)q0 < ref_n;
        const uint32_t b0 = R.pw ? 0u : R.byte(in0 ? q0 : 0);
        const uint32_t kc = kclass(d.pk);
        const uint32_t ll = dval_big(d, T, (int)kc);                         // LL x previous kind class
        if (d.bad || ll > blen - d.o) return DEC_ERR;
        if (ll) {
            uint32_t p1 = 16, p2 = 16;
            for (uint32_t j = 0; j < ll; j++) {
                int c;
                if (ll <= 8) c = C_LITR + (j == 0 ? (!in0 ? 4 : R.pw ? refbase(R, d.c0, d.d0, d.o) : refcode(b0, d.d0)) * 2 + 1
                                                  : refbase(R, d.c0, d.d0, d.o + j) * 2);
                else c = C_LIT2 + (p1 == 16 ? 16 : (int)((p2 == 16 ? p1 : p2 * 4 + p1) % 16));
                const uint32_t sy = dsym_small(d, T, c);
                uint32_t byte = sy < 4 ? (0x54474341u >> (8 * sy)) & 0xFFu : (uint32_t)'N';   // A C G T, N
                if (sy >= 5) byte = draw(d, 8);                                              // escape: a raw byte
                if (!sk.lit(d.o + j, (uint8_t)byte)) return DEC_ABORT;
                p2 = p1; p1 = sy < 4 ? sy : 0;
            }
            if (!sk.op(0, d.li, d.o, ll)) return DEC_ABORT;
            d.li += ll; d.o += ll;
        }
        if (d.o >= stop) break;
        const uint32_t kind = dsym_small(d, T, C_KIND + (int)(llc(ll) * 4 + kc));
        if (kind > K_FLIP) return DEC_ERR;
        // the kind's arguments, in stream order: at most one small symbol (REP: cache index - 1, ABS: strand, FLIP: cache
        // index), then one bucketed value (DELTA / REP / FLIP: zig-zag delta, SELF: distance) or, for ABS, 32 raw bits.
        // Each read appears once here, so the decoder's inlined code stays small (it shares the instruction cache).
        uint64_t p = 0;
        uint32_t sarg = 0, varg = 0;
        if (kind == K_REP || kind == K_ABS || kind == K_FLIP) sarg = dsym_small(d, T, kind == K_REP ? C_REPK : kind == K_ABS ? C_DIR : C_FLIPK);
        if (kind == K_ABS) p = draw(d, 32);
        else if (kind != K_CONT) varg = dval_big(d, T, kind == K_DELTA ? 4 + (ll == 0 ? 0 : 1) : kind == K_REP ? 6 : kind == K_SELF ? 7 : 14);
        const uint32_t dist = kind == K_SELF ? varg : 0;
        uint32_t dir = kind == K_ABS ? sarg : 0;
        const int ki = kind == K_REP ? 1 + (int)sarg : kind == K_FLIP ? (int)sarg : 0;
        const int32_t dd = (kind == K_DELTA || kind == K_REP || kind == K_FLIP) ? unzz(varg) : 0;
        if ((kind == K_REP || kind == K_FLIP) && ki >= d.nc) return DEC_ERR;
        const uint32_t L = dval_big(d, T, 8 + (int)kind) + MINL;            // LEN x kind
        if (d.bad || L > blen - d.o) return DEC_ERR;
        uint32_t okind; uint64_t osrc;
        if (kind == K_SELF) {
            if (dist == 0 || dist > d.o) return DEC_ERR;
            okind = 2; osrc = d.o - dist;
        } else {
            if (kind == K_FLIP) {
                uint64_t gc; uint32_t gd;
                dget(d, ki, gc, gd);
                dir = gd ^ 1;
                const int64_t e = (gd ? (int64_t)gc - (int64_t)d.o : (int64_t)gc + (int64_t)d.o) + dd;
                if (e < 0) return DEC_ERR;
                p = (uint64_t)e;
            } else if (kind != K_ABS) {
                uint64_t gc; uint32_t gd;
                dget(d, kind == K_REP ? ki : 0, gc, gd);
                dir = gd;
                const int64_t e = (gd ? (int64_t)gc - (int64_t)d.o - (int64_t)L + 1 : (int64_t)gc + (int64_t)d.o) + dd;
                if (e < 0) return DEC_ERR;
                p = (uint64_t)e;
            }
            if (p > ref_n || L > ref_n - p) return DEC_ERR;
            okind = dir ? 3 : 1; osrc = p;
            dpush(d, dir ? (uint64_t)((int64_t)p + (int64_t)L - 1 + (int64_t)d.o) : (uint64_t)((int64_t)p - (int64_t)d.o), dir);
        }
        if (!sk.op(okind, osrc, d.o, L)) return DEC_ABORT;
        d.o += L; d.pk = kind + 1;
    }
    if (d.o < blen || validated) return DEC_DONE;    // stopped inside a validated block, or at its end
    if (d.bad || d.x != RANS_L || d.st.left() != 0) return DEC_ERR;
    return DEC_DONE;
}

// keeps the ops and literals that fall inside [ox0, ox1) of the block
struct WindowSink {
    Op* ops; uint8_t* lits; uint32_t ox0, ox1, nops, nlits;
    template <class D> __device__ __forceinline__ void at(const D&) const {}
    __device__ bool more() const { return true; }
    __device__ bool lit(uint32_t o, uint8_t b) {
        if (o < ox0 || o >= ox1) return true;
        if (nlits >= LIT_CAP) return false;
        lits[nlits++] = b;
        return true;
    }
    __device__ bool op(uint32_t kind, uint64_t src, uint32_t dst, uint32_t len) {
        if (dst >= ox1 || dst + len <= ox0) return true;
        if (kind == 2 || nops >= OPS_CAP) return false;
        const uint32_t lo = dst > ox0 ? dst : ox0, hi = dst + len < ox1 ? dst + len : ox1;
        Op o; o.src = kind == 0 ? nlits - (hi - lo) : (uint32_t)src; o.dk = (uint16_t)(dst | (kind << 14)); o.len = (uint16_t)len;
        ops[nops++] = o;
        return true;
    }
};
// heavy path: literals straight into the block buffer, copies (up to ox1) into a chunk of HOPS ops
struct BlockSink {
    uint8_t* buf; Op* ops; uint32_t nops, ox1;
    template <class D> __device__ __forceinline__ void at(const D&) const {}
    __device__ bool more() const { return nops + 1 < (uint32_t)HOPS; }
    __device__ bool lit(uint32_t o, uint8_t b) { buf[o] = b; return true; }
    __device__ bool op(uint32_t kind, uint64_t src, uint32_t dst, uint32_t len) {
        if (kind == 0 || dst >= ox1) return true;
        Op o; o.src = (uint32_t)src; o.dk = (uint16_t)(dst | (kind << 14)); o.len = (uint16_t)len;
        ops[nops++] = o;
        return true;
    }
};

// ---------------------------------------------------------------- 16-byte register transforms
// Byte-parallel base classes on four bytes. code: A/a 0, C/c 1, G/g 2, T/t 3 for those letters (bits 1-2 of the
// ASCII code, x ^ x>>1); the mask keeps the bytes that really are one of the eight letters: each byte, lower-cased,
// is compared with the letter its code names ('a' 'c' 'g' 't' picked by a byte permute), with an exact zero-byte test.
__device__ __forceinline__ uint32_t acgt4(uint32_t w, uint32_t& t) {
    t = ((w >> 1) ^ (w >> 2)) & 0x03030303u;
    const uint32_t e = __byte_perm(0x74676361u, 0u, t | (t >> 12));   // letters for bytes 0, 2, 1, 3 (selector order)
    const uint32_t d = __byte_perm(w | 0x20202020u, 0u, 0x3120u) ^ e;  // the lower-cased bytes in that order
    uint32_t z = ~(((d & 0x7F7F7F7Fu) + 0x7F7F7F7Fu) | d) & 0x80808080u;   // 0x80 where a byte matched
    z = __byte_perm(z, 0u, 0x3120u);
    return (z >> 7) * 0xFFu;
}
__device__ __forceinline__ uint32_t comp4(uint32_t w) {        // ACGTacgt complemented, case kept (pv_v1.h:74-75)
    uint32_t t;
    const uint32_t m = acgt4(w, t);
    const uint32_t at = ~(t ^ (t >> 1)) & 0x01010101u;        // A and T (xor 0x15) vs C and G (xor 0x04)
    return w ^ ((0x04040404u + at * 0x11u) & m);
}
// tokens A/a 0, C/c 1, G/g 2, T/t 3, else 4 (pv_v1.h:76); of the complemented bytes when rc (3 - code)
__device__ __forceinline__ uint32_t tok4(uint32_t w, bool rc) {
    uint32_t t;
    const uint32_t m = acgt4(w, t);
    if (rc) t ^= 0x03030303u;
    return (t & m) | (0x04040404u & ~m);
}
__device__ __forceinline__ void rev16(uint32_t v[4]) {
    const uint32_t a = __byte_perm(v[3], 0, 0x0123), b = __byte_perm(v[2], 0, 0x0123), c = __byte_perm(v[1], 0, 0x0123),
                   d = __byte_perm(v[0], 0, 0x0123);
    v[0] = a; v[1] = b; v[2] = c; v[3] = d;
}
__device__ __forceinline__ uint32_t bytes_mask(int k0, int k1, int i) {   // bytes of word i inside [k0, k1)
    int lo = k0 - 4 * i, hi = k1 - 4 * i;
    lo = lo < 0 ? 0 : lo > 4 ? 4 : lo;
    hi = hi < 0 ? 0 : hi > 4 ? 4 : hi;
    if (lo >= hi) return 0;
    const uint32_t m = (hi - lo) == 4 ? 0xFFFFFFFFu : ((1u << (8 * (hi - lo))) - 1);
    return m << (8 * lo);
}
// L2 eviction priorities (createpolicy): evict_last for the reference spans the decode warms for the emission, so that
// the call's output stores do not push them out first; evict_first for the bytes the emission has read.
__device__ __forceinline__ uint64_t l2_evict_last() {
    uint64_t p;
    asm("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}
__device__ __forceinline__ uint64_t l2_evict_first() {
    uint64_t p;
    asm("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}
__device__ __forceinline__ uint4 ldg_hint(const uint4* q, uint64_t pol) {
    uint4 v;
    asm("ld.global.nc.L2::cache_hint.v4.u32 {%0, %1, %2, %3}, [%4], %5;" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(q), "l"(pol));
    return v;
}
// 16 bytes from any address (16-byte aligned loads on both sides, funnel-shifted); pol: an L2 policy for the loads,
// or 0
__device__ __forceinline__ void ldg16u(const uint8_t* p, uint32_t v[4], uint64_t pol = 0) {
    const uintptr_t a = (uintptr_t)p;
    const uint4* q = (const uint4*)(a & ~(uintptr_t)15);
    const uint32_t sh = (uint32_t)(a & 15);
    const uint4 lo = pol ? ldg_hint(q, pol) : __ldg(q), hi = pol ? ldg_hint(q + 1, pol) : __ldg(q + 1);   // (both, whatever the shift)
    const uint32_t w[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
    const uint32_t j = sh >> 2, b = (sh & 3) * 8;
    uint32_t y[6], x[5];                            // words j .. j + 4: shifted by two words, then by one
#pragma unroll
    for (int i = 0; i < 6; i++) y[i] = (j & 2) ? w[i + 2] : w[i];
#pragma unroll
    for (int i = 0; i < 5; i++) x[i] = (j & 1) ? y[i + 1] : y[i];
#pragma unroll
    for (int i = 0; i < 4; i++) v[i] = __funnelshift_r(x[i], x[i + 1], b);
}

// 16 bytes at any shared address (4-byte aligned loads, funnel-shifted; 4 readable bytes past the end)
__device__ __forceinline__ void lds16u(uint32_t a, uint32_t v[4]) {
    const uint32_t b = a & ~3u, sh = (a & 3u) * 8;
    uint32_t w[5];
#pragma unroll
    for (int i = 0; i < 5; i++) w[i] = lds32(b + 4 * i);
#pragma unroll
    for (int i = 0; i < 4; i++) v[i] = __funnelshift_r(w[i], w[i + 1], sh);
}
// the four letters of four 2-bit codes (8 bits) as bytes
__device__ __forceinline__ uint32_t letters4(uint32_t c8) {
    const uint32_t sel = (c8 & 3u) | ((c8 & 0xCu) << 2) | ((c8 & 0x30u) << 4) | ((c8 & 0xC0u) << 6);
    return __byte_perm(0x54474341u, 0u, sel);
}
// 16 bytes of the packed reference from position q (bytes outside [0, n) are 0, as the byte form's zero padding).
// Out of line and by value, so that the byte form's callers keep their vectors in registers.
__device__ __noinline__ uint4 packed16(const uint32_t* pw, const pv_ref_run* runs, const uint32_t* pidx, uint64_t n, int64_t q) {
    const RefView R{nullptr, n, 0, 0, 0, pw, runs, pidx};
    uint32_t v[4] = {0, 0, 0, 0};
    if (q < 0 || q + 16 > (int64_t)n) {
        for (int k = 0; k < 16; k++) {
            const int64_t x = q + k;
            const uint32_t b = (x >= 0 && x < (int64_t)n) ? R.packed_byte(x) : 0u;
            if (k < 4) v[0] |= b << (8 * k); else if (k < 8) v[1] |= b << (8 * (k - 4)); else if (k < 12) v[2] |= b << (8 * (k - 8)); else v[3] |= b << (8 * (k - 12));
        }
        return make_uint4(v[0], v[1], v[2], v[3]);
    }
    const uint32_t codes = __funnelshift_r(__ldg(pw + (q >> 4)), __ldg(pw + (q >> 4) + 1), (uint32_t)(q & 15) * 2);
#pragma unroll
    for (int i = 0; i < 4; i++) v[i] = letters4((codes >> (8 * i)) & 0xFFu);
    uint32_t i = __ldg(pidx + (q >> PV_REF_BUCKET_SHIFT));
    while (__ldg(&runs[i].start) + __ldg(&runs[i].len) <= (uint64_t)q) i++;
    for (; __ldg(&runs[i].start) < (uint64_t)q + 16; i++) {
        const int64_t rs = (int64_t)__ldg(&runs[i].start), re = rs + __ldg(&runs[i].len);
        const int k0 = (int)((rs > q ? rs : q) - q), k1 = (int)((re < q + 16 ? re : q + 16) - q);
        const uint32_t fill = __ldg(&runs[i].byte) * 0x01010101u;
#pragma unroll
        for (int w = 0; w < 4; w++) { const uint32_t m = bytes_mask(k0, k1, w); v[w] = (v[w] & ~m) | (fill & m); }
    }
    return make_uint4(v[0], v[1], v[2], v[3]);
}

// ---------------------------------------------------------------- gathers: raw block bytes [blo, blo + 16)
// 16 source bytes of op o for block offsets [blo, blo + 16), as if the op covered all of them (the caller keeps the
// bytes the op does cover). Literal bytes come from the item's literal array in shared memory (lits_sm: its address;
// the bytes around it are other fields of the slot, read but never used), reference bytes from the staged span or
// global memory, reverse-complement copies byte-reversed and complemented.
// Where an item's literal bytes are: in its shared slot (lits_sm, a shared address) or, for the emission kernel that
// reads decoded items in place, in the plan in global memory (lits_g).
// (rc: the cohort's reverse-complement reference, or NULL; pol: an L2 policy for the loads, or 0)
struct LitSrc { uint32_t sm; const uint8_t* g; const uint8_t* rc; uint64_t pol; };
// (one load path for every kind, its address chosen by selects - the lanes of a pass often hold ops of different
// kinds - then the byte reversal and complement of a reverse-complement copy)
template <bool LG>
__device__ __forceinline__ void op_src16(const Item* it, const RefView& R, const LitSrc& L, const Op& o, int64_t blo, uint32_t v[4]) {
    const int64_t dst = op_dst(o), len = o.len;
    const uint32_t kind = op_kind(o);
    const bool lit = kind == 0, rev = kind == 3;
    const int64_t q = rev ? (int64_t)o.src + len - 16 - (blo - dst) : (int64_t)o.src + (blo - dst);   // a copy's first byte
    const int64_t first = dst > (int64_t)it->ox0 ? dst : (int64_t)it->ox0;
    const int64_t li = (int64_t)o.src + (blo - first);                                                 // a literal's
    if (LG) {                                       // no span: literals and the byte reference from global memory
        if (L.rc) {                                 // (byte form) one load for every kind: a reverse-complement copy
            ldg16u(lit ? L.g + li : rev ? L.rc + ((int64_t)R.n - (int64_t)o.src - len + (blo - dst)) : R.g + q, v, L.pol);
            return;                                 // reads forward from the reverse-complement reference: done
        }
        if (lit || !R.pw) ldg16u(lit ? L.g + li : R.g + q, v, L.pol);
        else { const uint4 u = packed16(R.pw, R.runs, R.pidx, R.n, q); v[0] = u.x; v[1] = u.y; v[2] = u.z; v[3] = u.w; }
    } else {
        const bool in_span = lit || (q >= R.lo && q - R.lo + 16 <= (int64_t)R.len);
        const uint32_t sa = lit ? L.sm + (uint32_t)li : R.sm + (uint32_t)(q - R.lo);
        if (in_span) lds16u(sa, v);
        else if (R.pw) { const uint4 u = packed16(R.pw, R.runs, R.pidx, R.n, q); v[0] = u.x; v[1] = u.y; v[2] = u.z; v[3] = u.w; }
        else ldg16u(R.g + q, v);
    }
    if (rev) {
        rev16(v);
#pragma unroll
        for (int i = 0; i < 4; i++) v[i] = comp4(v[i]);
    }
}
struct BufGather {
    const Item* it; const uint8_t* buf;
    __device__ void operator()(int64_t blo, uint32_t r[4]) const {
        r[0] = r[1] = r[2] = r[3] = 0;
#pragma unroll
        for (int k = 0; k < 16; k++) {
            const int64_t q = blo + k;
            if (q >= (int64_t)it->ox0 && q < (int64_t)it->ox1) r[k >> 2] |= (uint32_t)buf[q] << (8 * (k & 3));
        }
    }
};

// a block served from the cohort's cache: its decoded bytes (the cache has 64 readable bytes around every row)
struct CacheGather {
    const uint8_t* blk;
    __device__ void operator()(int64_t blo, uint32_t r[4]) const { ldg16u(blk + blo, r); }
};

// lower-case mask of window positions [wp, wp + 16) (bit k = position wp + k)
// (the runs of an item with more than RUN_CAP of them, from global memory: rare, out of line)
__device__ __noinline__ uint32_t case_mask_global(const Item* it, const uint64_t* __restrict__ low, int64_t wp) {
    uint32_t m = 0;
    const int64_t x = (int64_t)it->s + wp;              // stream position of bit 0
    uint32_t lo = 0, hi = it->run_cnt;
    while (lo < hi) { const uint32_t mid = (lo + hi) >> 1; if ((int64_t)__ldg(low + 2 * (it->run_first + mid) + 1) <= x) lo = mid + 1; else hi = mid; }
    for (uint32_t r = lo; r < it->run_cnt; r++) {
        const int64_t rs = (int64_t)__ldg(low + 2 * (it->run_first + r)), re = (int64_t)__ldg(low + 2 * (it->run_first + r) + 1);
        if (rs >= x + 16) break;
        const int64_t a = rs > x ? rs : x, e = re < x + 16 ? re : x + 16;
        if (a < e) m |= ((1u << (e - a)) - 1) << (a - x);
    }
    return m;
}
__device__ __forceinline__ uint32_t case_mask(const Item* it, const uint64_t* __restrict__ low, int64_t wp) {
    if (it->run_cnt > (uint32_t)RUN_CAP) return case_mask_global(it, low, wp);
    uint32_t m = 0;
    for (uint32_t r = 0; r < it->run_cnt; r++) {
        const int64_t lo = it->runs[2 * r] > wp ? it->runs[2 * r] : wp;
        const int64_t hi = it->runs[2 * r + 1] < wp + 16 ? it->runs[2 * r + 1] : wp + 16;
        if (lo < hi) m |= ((1u << (hi - lo)) - 1) << (lo - wp);
    }
    return m;
}

// An item's output: row = its window's output row, [A, B) = the bytes of the row it writes, delta = window start -
// block start (block offset q is window position q - delta), rcw = the window is reverse-complemented. For the
// token-id output the addresses are element indices of out64 (as if it were a byte array at address 0), so the same
// 16-aligned chunking gives 16 ids per chunk, 16-byte aligned.
struct OutRange {
    uint8_t* row; uintptr_t A, B; int64_t delta; int rcw; bool cased;
};
__device__ __forceinline__ OutRange out_range(const Params& P, const Item* it) {
    OutRange g;
    const int64_t W = (int64_t)P.W;
    g.rcw = P.rc ? (P.rc[it->w] != 0) : 0;
    g.row = P.out64 ? (uint8_t*)(uintptr_t)((uint64_t)it->w * P.W) : P.out + (uint64_t)it->w * P.W;
    g.delta = (int64_t)it->s - (int64_t)it->bst;
    const int64_t wx0 = (int64_t)it->ox0 - g.delta, wx1 = (int64_t)it->ox1 - g.delta;
    g.A = (uintptr_t)(g.row + (g.rcw ? W - wx1 : wx0));
    g.B = (uintptr_t)(g.row + (g.rcw ? W - wx0 : wx1));
    g.cased = P.apply_case && !P.tokens && it->run_cnt;
    return g;
}
// the token-id store (pv_windows_ids): 16 tokens -> 16 int64 ids at element index ca of out64 (those in [A, B) when not
// whole). Out of line, with plain arguments, so the byte stores' hot loop stays small.
__device__ __noinline__ void store_ids(int64_t* out64, int64_t i0, int64_t i1, int64_t i2, int64_t i3, int64_t i4, uintptr_t A,
                                      uintptr_t B, uintptr_t ca, uint32_t v0, uint32_t v1, uint32_t v2, uint32_t v3, bool whole) {
    const uint32_t v[4] = {v0, v1, v2, v3};
#pragma unroll
    for (int k = 0; k < 16; k++) {
        const uint32_t t = (v[k >> 2] >> (8 * (k & 3))) & 7u;
        const int64_t id = t == 0 ? i0 : t == 1 ? i1 : t == 2 ? i2 : t == 3 ? i3 : i4;
        if (whole || (ca + k >= A && ca + k < B)) out64[ca + k] = id;
    }
}
// the 16 forward bytes v of window positions [wpf, wpf + 16) -> the output chunk at ca (16-byte aligned): lower-case
// runs, reverse complement, tokens, then one vector store (or, at the ends of the item's range, its bytes in [A, B))
__device__ __forceinline__ void put16(const Params& P, const Item* it, const OutRange& g, uintptr_t ca, int64_t wpf, uint32_t v[4], bool whole) {
    if (g.cased) {
        const uint32_t m = case_mask(it, P.C.low, wpf);
        if (m) {
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const uint32_t m4 = (m >> (4 * i)) & 15u;
                const uint32_t bm = (m4 & 1u) * 0xFFu | (m4 & 2u) * 0x7F80u | (m4 & 4u) * 0x3FC000u | (m4 & 8u) * 0x1FE00000u;
                v[i] |= bm & 0x20202020u;
            }
        }
    }
    if (P.tokens) {
#pragma unroll
        for (int i = 0; i < 4; i++) v[i] = tok4(v[i], g.rcw);
    } else if (g.rcw) {
#pragma unroll
        for (int i = 0; i < 4; i++) v[i] = comp4(v[i]);
    }
    if (g.rcw) rev16(v);
    if (P.out64) {
        store_ids(P.out64, P.ids[0], P.ids[1], P.ids[2], P.ids[3], P.ids[4], g.A, g.B, ca, v[0], v[1], v[2], v[3],
                  whole || (ca >= g.A && ca + 16 <= g.B));
        return;
    }
    if (whole || (ca >= g.A && ca + 16 <= g.B)) {
        __stcs((uint4*)ca, make_uint4(v[0], v[1], v[2], v[3]));      // streaming: the windows are not read here again
    } else {                                        // an end of the range: its bytes, whole words as words
        const int lo = ca < g.A ? (int)(g.A - ca) : 0, hi = ca + 16 > g.B ? (int)(g.B - ca) : 16;
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int a = lo > 4 * i ? lo : 4 * i, b = hi < 4 * i + 4 ? hi : 4 * i + 4;
            if (a == 4 * i && b == 4 * i + 4) *(uint32_t*)(ca + 4 * i) = v[i];
            else
                for (int k = a; k < b; k++) *(uint8_t*)(ca + k) = (uint8_t)(v[i] >> (8 * (k - 4 * i)));
        }
    }
}

// one item's output range in 16-byte chunks of the output row; lanes `lane` of `nl` share the chunks
template <class Gather>
__device__ void emit(const Params& P, const Item* it, const Gather& gather, int lane, int nl) {
    const OutRange g = out_range(P, it);
    const int64_t W = (int64_t)P.W;
    for (uintptr_t ca = (g.A & ~(uintptr_t)15) + 16 * (uintptr_t)lane; ca < g.B; ca += 16 * (uintptr_t)nl) {
        const int64_t opos = (int64_t)(ca - (uintptr_t)g.row);
        const int64_t wpf = g.rcw ? W - 16 - opos : opos;      // window position of the first forward byte
        uint32_t v[4];
        gather(wpf + g.delta, v);
        put16(P, it, g, ca, wpf, v, false);
    }
}

// a block served from the block cache: out of line (rare, and it would add a third copy of the store path to the
// kernels' instruction cache footprint)
__device__ __noinline__ void emit_cached(const Params& P, const Item* it, int lane) { emit(P, it, CacheGather{it->cptr}, lane, 32); }

// bytes j.. of 16 (j in 0..15) taken from u: the ops of an item tile its range in order, so each op that starts inside
// a chunk overwrites it from its start on, and the next one overwrites from its own start
__device__ __forceinline__ void merge_from(uint32_t v[4], const uint32_t u[4], int j) {
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int sh = j - 4 * i;
        const uint32_t m = sh <= 0 ? 0xFFFFFFFFu : sh >= 4 ? 0u : 0xFFFFFFFFu << (8 * sh);
        v[i] = (v[i] & ~m) | (u[i] & m);
    }
}

// A decoded item's output, op by op. The ops of an item tile its range [ox0, ox1) in order; in the output row each op
// covers a run of bytes (reversed in place for a reverse-complemented window). First (emit_op_chunks), for each op in
// turn (the same op for the whole warp, so every lane takes the same load path), the 16-byte chunks of the row wholly
// inside the op's bytes: the lanes share them, each chunk one 16-byte load of the op's source (the reference, the
// reverse-complement reference, the staged span or the literal bytes) and one 16-byte store after case / reverse
// complement / tokens in registers. Then (emit_boundary) the chunks the first pass left: those holding an op boundary,
// or an end of the item's range, off a 16-byte boundary - one lane each, its bytes gathered from every op it overlaps
// (the op covering its first byte, then each op starting inside it over it from its start). it: the item's header
// (shared slot); ops and literal bytes in the slot too, or (LG) read in place from the item's record in the plan;
// g = out_range(P, it).
template <bool LG>
__device__ __forceinline__ void emit_op_chunks(const Params& P, const Item* it, const OutRange& g, const Op* ops,
                                               const LitSrc& L, const RefView& R, int lane) {
    // offsets inside a window and a block fit 32 bits (W < 2^31, blocks <= 2^14 bases): the arithmetic is 32-bit, only
    // the chunk addresses are 64-bit
    const int32_t W = (int32_t)P.W, delta = (int32_t)g.delta, ox0 = (int32_t)it->ox0, ox1 = (int32_t)it->ox1;
    const intptr_t row = (intptr_t)(uintptr_t)g.row;
    const int nops = it->nops;
    // the item's ops, loaded once by the warp (lane j: ops j and j + 32) and broadcast op by op, so that the pass does
    // not wait on one dependent load per op
    uint2 r0 = make_uint2(0u, 0u), r1 = make_uint2(0u, 0u);
    if (lane < nops) r0 = *(const uint2*)(ops + lane);
    if (lane + 32 < nops) r1 = *(const uint2*)(ops + lane + 32);
    for (int k = 0; k < nops; k++) {
        const uint32_t ox = __shfl_sync(0xffffffffu, k < 32 ? r0.x : r1.x, k & 31);
        const uint32_t oy = __shfl_sync(0xffffffffu, k < 32 ? r0.y : r1.y, k & 31);
        Op o;
        o.src = ox; o.dk = (uint16_t)(oy & 0xFFFFu); o.len = (uint16_t)(oy >> 16);
        const int32_t d0 = (int32_t)op_dst(o) > ox0 ? (int32_t)op_dst(o) : ox0;
        const int32_t d1 = (int32_t)(op_dst(o) + o.len) < ox1 ? (int32_t)(op_dst(o) + o.len) : ox1;
        const int32_t lo = g.rcw ? W - (d1 - delta) : d0 - delta, hi = g.rcw ? W - (d0 - delta) : d1 - delta;   // its row bytes
        const intptr_t a0 = (row + lo + 15) & ~(intptr_t)15, a1 = (row + hi) & ~(intptr_t)15;
        if (LG && L.rc) {
            // the byte form read in place: whatever the op's kind, a chunk's source is one address per op plus the
            // chunk's window position - a literal's bytes in the plan, a copy's in the reference or, for a
            // reverse-complement copy, read forward in the reverse-complemented reference (op_src16's addresses)
            const uint32_t kind = op_kind(o);
            const intptr_t dst = (intptr_t)op_dst(o), len = (intptr_t)o.len, src = (intptr_t)o.src;
            const intptr_t base = kind == 0 ? (intptr_t)(uintptr_t)L.g + src - d0 + delta
                                : kind == 3 ? (intptr_t)(uintptr_t)L.rc + (intptr_t)R.n - src - len - dst + delta
                                            : (intptr_t)(uintptr_t)R.g + src - dst + delta;
            for (intptr_t c = a0 + 16 * (intptr_t)lane; c < a1; c += 16 * 32) {
                const int32_t ro = (int32_t)(c - row);
                const int32_t wpf = g.rcw ? W - 16 - ro : ro;
                uint32_t v[4];
                ldg16u((const uint8_t*)(uintptr_t)(base + wpf), v, L.pol);
                put16(P, it, g, (uintptr_t)c, wpf, v, true);
            }
            continue;
        }
        for (intptr_t c = a0 + 16 * (intptr_t)lane; c < a1; c += 16 * 32) {
            const int32_t ro = (int32_t)(c - row);
            const int32_t wpf = g.rcw ? W - 16 - ro : ro;
            uint32_t v[4];
            op_src16<LG>(it, R, L, o, wpf + delta, v);
            put16(P, it, g, (uintptr_t)c, wpf, v, true);
        }
    }
}
// Boundary b (0 .. nops) is the row offset where op b starts (b = 0: the range's first byte in window order) or, b =
// nops, where the range ends; its chunk is handled unless the boundary is 16-byte aligned in memory or the lane of
// boundary b - 1 already has that chunk.
template <bool LG>
__device__ __forceinline__ void emit_boundary(const Params& P, const Item* it, const OutRange& g, const Op* ops,
                                              const LitSrc& L, const RefView& R, int b) {
    const int32_t W = (int32_t)P.W, delta = (int32_t)g.delta, ox0 = (int32_t)it->ox0, ox1 = (int32_t)it->ox1;
    const intptr_t row = (intptr_t)(uintptr_t)g.row;
    const int nops = it->nops;
    const int32_t wb = b == 0 ? ox0 - delta : b == nops ? ox1 - delta : (int32_t)op_dst(ops[b]) - delta;   // window position
    const int32_t ob = g.rcw ? W - wb : wb;        // the boundary's row offset (a reversed row: its end there)
    const intptr_t ab = row + ob;
    const int32_t wprev = b == 0 ? 0 : b - 1 == 0 ? ox0 - delta : (int32_t)op_dst(ops[b - 1]) - delta;
    const intptr_t aprev = row + (g.rcw ? W - wprev : wprev);
    if ((ab & 15) == 0 || (b > 0 && (aprev & ~(intptr_t)15) == (ab & ~(intptr_t)15) && (aprev & 15) != 0)) return;
    const intptr_t c = ab & ~(intptr_t)15;
    const int32_t ro = (int32_t)(c - row);
    const int32_t wpf = g.rcw ? W - 16 - ro : ro;
    const int32_t blo = wpf + delta;
    const int32_t klo = blo > ox0 ? blo : ox0, khi = blo + 16 < ox1 ? blo + 16 : ox1;
    if (klo >= khi) return;
    int k = 0, hk = nops;                       // the op covering klo: the first ending after it
    while (k < hk) {
        const int m = (k + hk) >> 1;
        if ((int32_t)(op_dst(ops[m]) + ops[m].len) <= klo) k = m + 1; else hk = m;
    }
    if (k >= nops) return;
    uint32_t v[4];
    op_src16<LG>(it, R, L, ops[k], blo, v);
    for (int kk = k + 1; kk < nops; kk++) {
        const Op q = ops[kk];
        const int32_t dst = (int32_t)op_dst(q);
        if (dst >= khi) break;
        uint32_t u[4];
        op_src16<LG>(it, R, L, q, blo, u);
        merge_from(v, u, dst - blo);
    }
    put16(P, it, g, (uintptr_t)c, wpf, v, false);
}
template <bool LG>
__device__ void emit_ops(const Params& P, const Item* it, const Op* ops, const LitSrc& L, const RefView& R, int lane) {
    const OutRange g = out_range(P, it);
    emit_op_chunks<LG>(P, it, g, ops, L, R, lane);
    for (int b = lane; b <= (int)it->nops; b += 32) emit_boundary<LG>(P, it, g, ops, L, R, b);
}

// ---------------------------------------------------------------- TMA bulk copies and the mbarrier they complete on
__device__ __forceinline__ void mbar_init(uint32_t bar) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" :: "r"(bar) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" :: "r"(bar), "r"(bytes) : "memory");
}
// one try: the thread is suspended until the phase completes or about WAIT_TRY_NS have passed (so a waiting lane
// issues a handful of instructions per microsecond, not a spin loop's worth)
constexpr uint32_t WAIT_TRY_NS = 1000;
__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t phase) {
    uint32_t ok;
    asm volatile("{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3; selp.u32 %0, 1, 0, p; }"
                 : "=r"(ok) : "r"(bar), "r"(phase), "n"(WAIT_TRY_NS) : "memory");
    return ok != 0;
}
// global -> shared, 16-byte aligned addresses and a multiple of 16 bytes, completing on `bar`
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 :: "r"(dst), "l"(src), "r"(bytes), "r"(bar) : "memory");
}
constexpr uint32_t WAIT_SPINS = 1u << 13;   // tries of a bounded wait on a bulk copy (milliseconds); then status 4
constexpr uint32_t TEST_WAIT_SPINS = 1u << 6;   // the same under PV_WIN_TEST_WAIT, so the test's wait expires soon
constexpr uint32_t DRAIN_SPINS = 1u << 20;  // after an expired wait: the bound on waiting for the copies to land (~1 s)

// Programmatic dependent launch: the window kernels are launched so that their CTAs may be scheduled while the kernel
// before them on the stream is still running; each waits here, before it reads anything that kernel wrote, until it
// has completed and its memory is visible (a no-op when launched without the attribute). The kernels whose successors
// can start early say so as soon as they start.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---------------------------------------------------------------- items
constexpr int WARPS = 4;                     // one item per warp
// A warp's shared slot: its Item, then its assembly's decode table (tab_area bytes: the cohort's largest table), then
// its block's stream (pay_cap bytes; a longer stream is read from global memory).
__device__ __forceinline__ Item* slot_item(uint8_t* slot) { return (Item*)slot; }
__device__ __forceinline__ uint8_t* slot_tab(const Params& P, uint8_t* slot) { (void)P; return slot + sizeof(Item); }
__device__ __forceinline__ uint8_t* slot_pay(const Params& P, uint8_t* slot) { return slot + sizeof(Item) + P.tab_area; }
__device__ __forceinline__ uint8_t* slot_span(const Params& P, uint8_t* slot) { return slot + sizeof(Item) + P.tab_area + P.pay_cap; }
constexpr int SPAN_MARGIN = 64;              // reference bases staged on each side of the block's start diagonal
// PK / CP: the cohort keeps the packed reference / the compact block table. The kernels are instantiated per form, so
// the plain form's code carries neither (smaller code for the instruction cache, no runtime checks).
template <bool PK>
__device__ __forceinline__ RefView slot_ref(const Params& P, uint8_t* slot) {
    const Item* it = slot_item(slot);
    return RefView{P.C.ref, P.C.ref_n, it->span_lo, it->span_len, smem_addr(slot_span(P, slot)),
                   PK ? P.C.pref : nullptr, P.C.pruns, P.C.pidx};
}

// lane 0: the item's window, block and cell (items of a window are the cells [jS, (j+1)S) of the cohort's checkpoint
// stride S it touches, S = Q without an index, so then one item per block), its nominal output range (cell and window
// intersected); false when there is nothing to decode
__device__ bool item_locate(const Params& P, uint64_t item, Item* it) {
    it->state = ST_IDLE;
    it->nops = 0; it->nlits = 0;
    if (item >= P.total) return false;
    it->idx = item;
    const uint64_t w = item < 0xFFFFFFFFull ? (uint64_t)((uint32_t)item / (uint32_t)P.bpw) : item / P.bpw, j = item - w * P.bpw;
    const int64_t a = P.wasm[w], s = P.wstart[w];
    const pv_dev_cohort& C = P.C;
    if (a < 0 || a >= C.nasm) { if (j == 0) report(P, w, PV_STATUS_WINDOW); return false; }
    const pv_asm_rec& R = C.asms[a];
    if (s < 0 || (uint64_t)s + P.W > R.nbases) { if (j == 0) report(P, w, PV_STATUS_WINDOW); return false; }
    const uint32_t cs = P.cshift;
    const uint64_t Q = C.Q, g0 = (uint64_t)s >> cs, g1 = ((uint64_t)s + P.W - 1) >> cs, g = g0 + j;
    if (g > g1) return false;
    const uint64_t b = g >> (P.qshift - cs);
    const uint64_t bst = b * Q, blen = R.nbases - bst < Q ? R.nbases - bst : Q;
    const uint64_t x0 = (uint64_t)s > bst ? (uint64_t)s : bst, x1 = (uint64_t)s + P.W < bst + blen ? (uint64_t)s + P.W : bst + blen;
    it->w = (int64_t)w; it->s = (uint64_t)s; it->bst = bst; it->gblk = R.blk_base + b; it->a = (int32_t)a;
    it->grp = R.grp_base + (b >> 5); it->gj = (uint32_t)(b & 31);
    it->gm = (uint32_t)(R.nb - (b & ~31ull) < 32 ? R.nb - (b & ~31ull) : 32);
    it->staged = 0;
    it->tab_off = R.tab_off; it->tab_bytes = (uint32_t)R.tab_bytes; it->span_lo = 0; it->span_len = 0;
    it->jc = (uint32_t)(g - (b << (P.qshift - cs)));
    it->wx0 = (uint32_t)(x0 - bst); it->wx1 = (uint32_t)(x1 - bst); it->blen = (uint32_t)blen;
    const uint32_t cx0 = it->jc << cs, cx1 = cx0 + (1u << cs);
    it->ox0 = it->wx0 > cx0 ? it->wx0 : cx0; it->ox1 = it->wx1 < cx1 ? it->wx1 : cx1;
    it->ck = NO_CK; it->co = 0;
    it->run_first = 0; it->run_cnt = 0; it->nops = 0; it->nlits = 0;
    it->state = ST_LOCATED;
    return true;
}

// lane 0, for a located item of a cohort with a checkpoint index: its decode starts at its cell's checkpoint j (the
// last event boundary at or before the cell's start), and its output range is what the decode from there produces up
// to the next cell's checkpoint - or, for the window's last cell of the block, up to the window's end - intersected
// with the window: [max(wx0, o_j), j last ? wx1 : o_j+1). So the items of a window tile it exactly, each event is
// decoded once (but the one reaching the window's end), and a long event spanning several cells belongs to one item.
// A block the index found corrupt reports status 1 (ST_ERR); an empty range leaves the item idle.
__device__ void item_ckpt(const Params& P, Item* it) {
    const pv_dev_cohort& C = P.C;
    const uint32_t ncs = P.qshift - P.cshift;
    const uint64_t k = (it->gblk << ncs) + it->jc;
    const pv_ckpt* ck = C.ckpt + k;
    const uint32_t ow = __ldg((const uint32_t*)ck + 7);            // o | flags << 16
    if (ow & (PV_CKPT_BAD << 16)) { it->state = ST_ERR; report(P, it->w, PV_STATUS_DECODE); return; }
    if (ow & (PV_CKPT_CACHED << 16)) {              // (reached when the block table was not read): the cell range
        it->state = ST_CACHED;
        it->cptr = C.cache + (uint64_t)__ldg((const uint32_t*)ck + 1) * C.Q;
        return;
    }
    const uint32_t o0 = ow & 0xFFFFu;
    const bool last = it->jc == ((it->wx1 - 1) >> P.cshift);
    uint32_t o1 = it->wx1;
    if (!last) {
        const uint32_t on = it->jc + 1 < (1u << ncs) ? (__ldg((const uint32_t*)(ck + 1) + 7) & 0xFFFFu) : it->blen;
        o1 = on < o1 ? on : o1;
    }
    it->ox0 = it->wx0 > o0 ? it->wx0 : o0;
    it->ox1 = o1;
    if (it->ox0 >= it->ox1) { it->state = ST_IDLE; return; }
    it->ck = k; it->co = o0;
    it->cpos = ck_pos(__ldg((const uint32_t*)ck + 1), ow);
    const uint4 b = __ldg((const uint4*)ck + 1);
    const uint32_t lo = __ldg((const uint32_t*)ck + 2);
    it->cst = (int64_t)(ck_diag(lo, b.z) << 1) | (int64_t)((b.z >> 7) & 1u);
}

// one lane: the lower-case runs overlapping the item's output range, from r0, the block's first run (C.brun)
__device__ __noinline__ void item_runs_from(const Params& P, Item* it, uint32_t r0) {
    const pv_dev_cohort& C = P.C;
    const pv_asm_rec& R = C.asms[it->a];
    it->run_cnt = 0;
    if (!(P.apply_case && !P.tokens && R.low_cnt)) return;
    const uint64_t x0 = it->bst + it->ox0, x1 = it->bst + it->ox1, s = it->s;
    const uint64_t* low = C.low + 2 * R.low_base;
    uint64_t lo = r0;
    if (!C.brun) {
        uint64_t hi = R.low_cnt;
        lo = 0;
        while (lo < hi) { const uint64_t m = (lo + hi) >> 1; if (__ldg(low + 2 * m + 1) <= x0) lo = m + 1; else hi = m; }
    }
    while (lo < R.low_cnt && __ldg(low + 2 * lo + 1) <= x0) lo++;
    uint64_t e = lo;
    while (e < R.low_cnt && __ldg(low + 2 * e) < x1) e++;
    it->run_first = (uint32_t)(R.low_base + lo); it->run_cnt = (uint32_t)(e - lo);
    if (e - lo <= (uint64_t)RUN_CAP)
        for (uint64_t r = lo; r < e; r++) {
            const uint64_t rs = __ldg(low + 2 * r), re = __ldg(low + 2 * r + 1);
            it->runs[2 * (r - lo)] = (int32_t)((rs > x0 ? rs : x0) - s);
            it->runs[2 * (r - lo) + 1] = (int32_t)((re < x1 ? re : x1) - s);
        }
}
// lane 0: the lower-case runs overlapping the item's output range (window-relative, clipped to it)
__device__ void item_runs(const Params& P, Item* it) {
    const pv_dev_cohort& C = P.C;
    const pv_asm_rec& R = C.asms[it->a];
    if (!(P.apply_case && !P.tokens && R.low_cnt)) return;
    const uint64_t x0 = it->bst + it->ox0, x1 = it->bst + it->ox1, s = it->s;
    const uint64_t* low = C.low + 2 * R.low_base;
    uint64_t lo = 0;
    if (C.brun) {                                   // from the block's first run, a step or two
        lo = __ldg(C.brun + it->gblk);
        while (lo < R.low_cnt && __ldg(low + 2 * lo + 1) <= x0) lo++;
    } else {
        uint64_t hi = R.low_cnt;
        while (lo < hi) { const uint64_t m = (lo + hi) >> 1; if (__ldg(low + 2 * m + 1) <= x0) lo = m + 1; else hi = m; }
    }
    uint64_t e = lo;
    while (e < R.low_cnt && __ldg(low + 2 * e) < x1) e++;
    it->run_first = (uint32_t)(R.low_base + lo); it->run_cnt = (uint32_t)(e - lo);
    if (e - lo <= (uint64_t)RUN_CAP)
        for (uint64_t r = lo; r < e; r++) {
            const uint64_t rs = __ldg(low + 2 * r), re = __ldg(low + 2 * r + 1);
            it->runs[2 * (r - lo)] = (int32_t)((rs > x0 ? rs : x0) - s);
            it->runs[2 * (r - lo) + 1] = (int32_t)((re < x1 ? re : x1) - s);
        }
}

// The block's stream (offset, length) and start state, into the Item; the state becomes ST_CACHED for a block served
// from the cache and ST_ERR for a stream too long to be valid. All lanes call it: the full table is read by lane 0;
// the compact table (the reference's CompactTab::get, pv_compact.h:37-48, a pass over up to 31 earlier blocks of the
// group) is read by the warp at once: lane k holds block k of the group, the offset is a masked sum of the earlier
// lengths and the state a masked sum of the chain increments since the last absolute state (the group's first block
// or an exception).
template <bool CP>
__device__ void item_block(const Params& P, Item* it, int lane) {
    const pv_dev_cohort& C = P.C;
    if (!CP) {
        if (lane != 0) return;
        const uint64_t loc = __ldg(C.blocks + 2 * it->gblk);
        it->pst = it->cst = (int64_t)__ldg(C.blocks + 2 * it->gblk + 1);
        it->poff = loc_off(loc);
        it->plen = loc_len(loc);
        if (it->plen == (uint32_t)PV_BLOCK_CACHED) { it->state = ST_CACHED; it->cptr = C.cache + loc_off(loc) * C.Q; }
        else if (it->plen == (uint32_t)PV_BLEN_BAD) { it->state = ST_ERR; report(P, it->w, PV_STATUS_DECODE); }
        return;
    }
    const uint32_t j = it->gj, m = it->gm;
    const pv_blk_group* G = C.groups + it->grp;
    const uint64_t goff = __ldg(&G->off);
    const int64_t gst = __ldg(&G->state);
    const uint32_t emask = __ldg(&G->exc_mask), ebase = __ldg(&G->exc_base);
    const uint32_t v = (uint32_t)lane < m ? __ldg(C.btab + (it->gblk - j) + lane) : 0u;
    const uint32_t len = v & 0xFFFFu;
    const int32_t code = (int32_t)(int16_t)(v >> 16);
    const uint64_t off = goff + __reduce_add_sync(0xffffffffu, (uint32_t)lane < j ? len : 0u);
    const int b = 31 - __clz((emask | 1u) & ((2u << j) - 1u));        // the last absolute state at or before block j
    const int64_t base = b == 0 ? gst : __ldg(C.bexc + ebase + __popc(emask & ((1u << b) - 1u)));
    const int32_t cprev = __shfl_up_sync(0xffffffffu, code, 1);
    const uint32_t dprev = lane - 1 == b ? (uint32_t)(base & 1) : (uint32_t)(cprev & 1);
    const int32_t inc = (lane > b && (uint32_t)lane <= j) ? (dprev ? -(int32_t)C.Q : (int32_t)C.Q) + (code >> 1) : 0;
    const int32_t sum = (int32_t)__reduce_add_sync(0xffffffffu, (uint32_t)inc);
    const int32_t cj = __shfl_sync(0xffffffffu, code, (int)j);
    const uint32_t lj = __shfl_sync(0xffffffffu, len, (int)j);
    if (lane != 0) return;
    const int64_t c = (base >> 1) + sum;
    const uint32_t dir = (int)j == b ? (uint32_t)(base & 1) : (uint32_t)(cj & 1);
    it->poff = off; it->plen = lj; it->pst = it->cst = (int64_t)((uint64_t)c << 1) | (int64_t)dir;
    const uint32_t cmask = __ldg(&G->cache_mask);
    if ((cmask >> j) & 1u) {
        it->state = ST_CACHED;
        it->cptr = C.cache + (uint64_t)(__ldg(&G->cache_base) + __popc(cmask & ((1u << j) - 1u))) * C.Q;
    }
}

// the reference span of an item, 16-byte aligned: the diagonal current where its decode starts (the block's start
// diagonal, or its checkpoint's) over the range its decode covers, or (out_only) under the item's output range only,
// with a margin either way; empty when it would not fit `cap` bytes
__device__ __forceinline__ void item_span(const Params& P, Item* it, bool out_only, uint64_t cap) {
    const int64_t st = it->cst, c0 = st >> 1;
    const bool ck = it->ck != NO_CK;               // from a checkpoint the decode covers [co, ox1), else the whole block
    const int64_t o0 = out_only ? (int64_t)it->ox0 : (int64_t)it->co, o1 = (out_only || ck) ? (int64_t)it->ox1 : (int64_t)it->blen;
    int64_t lo = (st & 1) ? c0 - o1 + 1 - SPAN_MARGIN : c0 + o0 - SPAN_MARGIN, hi = (st & 1) ? c0 - o0 + 1 + SPAN_MARGIN : c0 + o1 + SPAN_MARGIN;
    lo = lo < 0 ? 0 : lo; hi = hi > (int64_t)P.C.ref_n ? (int64_t)P.C.ref_n : hi;
    uint64_t ra = 0, re = 0;
    if (lo < hi) { ra = (uint64_t)lo & ~15ull; re = ((uint64_t)hi + 15) & ~15ull; }
    if (re - ra + 16 > cap) re = ra;
    it->span_lo = (int64_t)ra; it->span_len = (uint32_t)(re - ra);
}

// lane 0: the reference span the decode's starting diagonal covers over the range it decodes, with a margin (the
// literal contexts and most copy sources read it from shared memory), then TMA bulk copies into the warp's slot of the
// assembly's decode table, the block's stream when it fits and, for the byte reference, the span
template <bool PK>
__device__ void item_stage(const Params& P, uint8_t* slot, uint32_t bar) {
    Item* it = slot_item(slot);
    const pv_dev_cohort& C = P.C;
    if (it->ck != NO_CK) {
        // from a checkpoint: the decode covers [co, ox1), little more than the output range
        item_span(P, it, false, P.span_cap);
        if (!it->span_len) item_span(P, it, true, P.span_cap);
    } else if (P.narrow) {
        // windows shorter than a block: the slot holds the diagonal under the output range only (what the emission
        // reads); the whole block's span is warmed in L2 for the literal contexts the decode reads off it
        item_span(P, it, false, ~0ull);
        if (!PK && it->span_len)
            asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" :: "l"(C.ref + it->span_lo), "r"(it->span_len) : "memory");
        item_span(P, it, true, P.span_cap);
    } else {
        item_span(P, it, false, P.span_cap);
    }
    const uint64_t ra = (uint64_t)it->span_lo;
    const uint8_t* src = C.payload + it->poff;
    const uintptr_t pa = (uintptr_t)src & ~(uintptr_t)15, pe = ((uintptr_t)src + it->plen + 15) & ~(uintptr_t)15;
    it->staged = pe - pa <= (uintptr_t)P.pay_cap;
    const uint32_t span_tma = PK ? 0u : it->span_len;
    mbar_init(bar);
    mbar_expect(bar, it->tab_bytes + (it->staged ? (uint32_t)(pe - pa) : 0u) + span_tma + (P.test_wait ? 16u : 0u));
    bulk_g2s(smem_addr(slot_tab(P, slot)), C.tabs + it->tab_off, it->tab_bytes, bar);
    if (it->staged) bulk_g2s(smem_addr(slot_pay(P, slot)), (const void*)pa, (uint32_t)(pe - pa), bar);
    if (span_tma) bulk_g2s(smem_addr(slot_span(P, slot)), C.ref + ra, span_tma, bar);
}

// the warp: the span unpacked from the packed reference into the slot (16 bases a lane-step), then the runs of other
// bytes that overlap it written over
__device__ void stage_span_packed(const Params& P, uint8_t* slot, int lane) {
    const Item* it = slot_item(slot);
    const pv_dev_cohort& C = P.C;
    const uint64_t lo = (uint64_t)it->span_lo, hi = lo + it->span_len;
    uint8_t* sp = slot_span(P, slot);
    for (uint32_t i = lane; i < it->span_len / 16; i += 32) {
        const uint32_t w = __ldg(C.pref + (lo >> 4) + i);
        *(uint4*)(sp + 16 * i) = make_uint4(letters4(w & 0xFFu), letters4((w >> 8) & 0xFFu), letters4((w >> 16) & 0xFFu), letters4(w >> 24));
    }
    __syncwarp();
    if (lo >= hi) return;
    uint32_t r = __ldg(C.pidx + (lo >> PV_REF_BUCKET_SHIFT));
    while (__ldg(&C.pruns[r].start) + __ldg(&C.pruns[r].len) <= lo) r++;
    for (; __ldg(&C.pruns[r].start) < hi; r++) {
        const uint64_t rs = __ldg(&C.pruns[r].start), re = rs + __ldg(&C.pruns[r].len);
        const uint8_t byte = (uint8_t)__ldg(&C.pruns[r].byte);
        for (uint64_t x = (rs > lo ? rs : lo) + lane; x < (re < hi ? re : hi); x += 32) sp[x - lo] = byte;
    }
}

// lane 0: wait, bounded, for the slot's bulk copies to complete on `bar` (phase 0). If the wait expires the window
// reports status 4 (the reference's expired wait, pv_cuda.cu:26,78) and the item is dropped, and lane 0 then waits on,
// bounded again, until the copies have landed: a CTA must not leave while a copy still targets its shared memory.
// Under PV_WIN_TEST_WAIT the barrier expects 16 bytes that no copy brings, so the first wait expires for sure; a
// 16-byte copy issued then completes them, and the second wait ends once every copy, that one included, has landed.
enum { WAIT_OK = 0, WAIT_EXPIRED = 1, WAIT_STUCK = 2 };   // STUCK: a copy may still land in the slot; do not reuse it
// (phase: the parity of the barrier phase the copies complete; a barrier initialised once and used for one item after
// another alternates 0, 1, 0, ...)
__device__ int slot_wait_ex(const Params& P, Item* it, uint32_t bar, uint32_t phase = 0) {
    const uint32_t lim = P.test_wait ? TEST_WAIT_SPINS : WAIT_SPINS;
    for (uint32_t k = 0; k < lim; k++)
        if (mbar_try(bar, phase)) return WAIT_OK;
    report(P, it->w, PV_STATUS_WAIT);
    it->state = ST_ERR;
    if (P.test_wait) bulk_g2s(smem_addr(&it->landing), P.C.tabs, 16, bar);
    for (uint32_t k = 0; k < DRAIN_SPINS; k++)
        if (mbar_try(bar, phase)) return WAIT_EXPIRED;
    return WAIT_STUCK;
}
__device__ bool slot_wait(const Params& P, Item* it, uint32_t bar) { return slot_wait_ex(P, it, bar, 0) == WAIT_OK; }

// lane 0 of the item's warp: wait (bounded) for the slot's copies, then decode the block keeping the window's ops
template <bool PK>
__device__ void item_decode(const Params& P, uint8_t* slot, uint32_t bar) {
    Item* it = slot_item(slot);
    if (!slot_wait(P, it, bar)) return;
    trace_at(P, it->idx, 2);
    if (P.force_block || !it->staged) { it->state = ST_HEAVY; return; }   // (a stream longer than the slot: uncached long block)
    WindowSink sk{it->ops, it->lits, it->ox0, it->ox1, 0, 0};
    const uint32_t sp = smem_addr(slot_pay(P, slot)) + (uint32_t)((uintptr_t)(P.C.payload + it->poff) & 15);
    Dec<SmemStream> d;
    uint32_t stop = it->blen;
    if (it->ck != NO_CK) { dec_init_ck(d, SmemStream{sp + (uint32_t)(it->cpos - it->poff), sp + it->plen}, P.C.ckpt + it->ck); stop = it->ox1; }
    else dec_init(d, SmemStream{sp, sp + it->plen}, it->pst);
    const int r = decode_events(d, SmemTab{smem_addr(slot_tab(P, slot))}, slot_ref<PK>(P, slot), it->blen, stop, sk, it->ck != NO_CK);
    trace_at(P, it->idx, 3);
    it->nops = (uint16_t)sk.nops; it->nlits = (uint16_t)sk.nlits;
    if (r == DEC_DONE) it->state = ST_OK;
    else if (r == DEC_ABORT) it->state = ST_HEAVY;
    else { it->state = ST_ERR; report(P, it->w, PV_STATUS_DECODE); }
}

// the CTA decodes a heavy item into its shared block buffer, ops in order, then emits it. Out of line: it is rare, and
// its code (a second decoder and an emission) would otherwise share the instruction cache with the common path. The
// assembly's table: staged in the slot (fused kernel), or read through L1 (GT: the emission kernel, whose slots leave
// the table out so that more of them fit)
template <bool PK, bool GT>
__device__ __noinline__ void heavy_item(const Params& P, uint8_t* slot, uint8_t* buf, Op* hops) {
    __shared__ int h_res, h_nops;
    __shared__ Dec<GlobalStream> h_dec;
    const Item* it = slot_item(slot);
    const pv_dev_cohort& C = P.C;
    using Tab = typename std::conditional<GT, GlobalTab, SmemTab>::type;
    Tab T;
    if constexpr (GT) T.b = C.tabs + it->tab_off; else T.b = smem_addr(slot_tab(P, slot));
    const RefView R = slot_ref<PK>(P, slot);
    if (threadIdx.x == 0) {
        const uint8_t* src = C.payload + it->poff;
        dec_init(h_dec, GlobalStream{src, src + it->plen}, it->pst);
    }
    for (;;) {
        __syncthreads();
        if (threadIdx.x == 0) {
            Dec<GlobalStream> d = h_dec;
            BlockSink sk{buf, hops, 0, it->ox1};
            h_res = decode_events(d, T, R, it->blen, it->blen, sk);
            h_nops = (int)sk.nops;
            h_dec = d;
        }
        __syncthreads();
        const int nops = h_nops;
        for (int k = 0; k < nops; k++) {
            const Op o = hops[k];
            const uint32_t dst = op_dst(o), len = o.len, kind = op_kind(o);
            if (kind == 1) {
                for (uint32_t i = threadIdx.x; i < len; i += CTA) buf[dst + i] = (uint8_t)R.byte((int64_t)o.src + i);
            } else if (kind == 3) {
                for (uint32_t i = threadIdx.x; i < len; i += CTA) buf[dst + i] = comp_up((uint8_t)R.byte((int64_t)o.src + len - 1 - i));
            } else {
                const uint32_t dist = dst - o.src;
                for (uint32_t c = 0; c < len;) {
                    const uint32_t step = dist < len - c ? dist : len - c;
                    for (uint32_t i = threadIdx.x; i < step; i += CTA) buf[dst + c + i] = buf[o.src + c + i];
                    __syncthreads();
                    c += step;
                }
            }
            __syncthreads();
        }
        if (h_res != DEC_PAUSE) break;
    }
    if (h_res != DEC_DONE) {
        if (threadIdx.x == 0) report(P, it->w, PV_STATUS_DECODE);
        __syncthreads();
        return;
    }
    emit(P, it, BufGather{it, buf}, threadIdx.x, CTA);
    __syncthreads();
}

template <bool PK, bool CP>
__global__ void __launch_bounds__(CTA, 6) pv_windows_kernel(const __grid_constant__ Params P) {
    extern __shared__ uint4 smem_raw[];
    __shared__ __align__(8) uint64_t bars[WARPS];
    __shared__ Op hops[HOPS];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    pdl_wait();
    uint8_t* slot = (uint8_t*)smem_raw + (size_t)warp * P.slot_bytes;
    Item* it = slot_item(slot);
    const uint64_t item = (uint64_t)blockIdx.x * WARPS + warp;
    const uint32_t bar = smem_addr(&bars[warp]);
    if (lane == 0) {
        if (item < P.total) trace_at(P, item, 0);
        item_locate(P, item, it);
    }
    __syncwarp();
    if (it->state == ST_LOCATED) {
        item_block<CP>(P, it, lane);
        __syncwarp();
        if (lane == 0) {
            if (P.C.ckpt && it->state == ST_LOCATED) item_ckpt(P, it);
            if (it->state == ST_LOCATED || it->state == ST_CACHED) item_runs(P, it);
            trace_at(P, it->idx, 1);
        }
        __syncwarp();
        if (it->state == ST_LOCATED) {
            if (lane == 0) item_stage<PK>(P, slot, bar);
            __syncwarp();
            if (PK) stage_span_packed(P, slot, lane);
            __syncwarp();
            if (lane == 0) item_decode<PK>(P, slot, bar);
        }
    }
    __syncwarp();
    if (it->state == ST_OK) emit_ops<false>(P, it, it->ops, LitSrc{smem_addr(it->lits), nullptr, nullptr, 0}, slot_ref<PK>(P, slot), lane);
    else if (it->state == ST_CACHED) emit_cached(P, it, lane);
    __syncwarp();
    if (lane == 0 && item < P.total && it->state != ST_HEAVY) trace_done(P, it, 1);
    __syncthreads();
    uint8_t* buf = P.work + (uint64_t)blockIdx.x * P.C.Q;
    for (int t = 0; t < WARPS; t++) {
        uint8_t* sl = (uint8_t*)smem_raw + (size_t)t * P.slot_bytes;
        if (slot_item(sl)->state == ST_HEAVY) {
            heavy_item<PK, false>(P, sl, buf, hops);
            if (threadIdx.x == 0) trace_done(P, slot_item(sl), 1);
        }
    }
}

// ---------------------------------------------------------------- the split pipeline: decode lanes, then emission warps
// pv_decode_kernel: one item per LANE. Each lane locates its window and block, looks the block up, warms L2 with the
// reference span its emission will stage, and decodes its block's stream from global memory with its assembly's table
// read through L1 - so a warp runs 32 independent rANS chains at once instead of one (their latencies overlap inside
// the warp, and the other 31 lanes no longer idle). The result, the Item (ops and literal bytes inside the window),
// goes to the plan array in global memory. pv_emit_kernel: one item per WARP, as the fused kernel's emission.

// One lane's block lookup: pooled block gblk (block b of its assembly, whose first compact group is grp_base) -> its
// stream's payload offset and length, its start state c << 1 | dir, and (cache) its row in the block cache, or NULL.
// The compact table is walked as the reference's chain (pv_compact.h:40-46): offset and state of block j of its group.
struct BlockRec { uint64_t poff; int64_t pst; uint32_t plen; const uint8_t* cache; };
template <bool CP>
__device__ __forceinline__ BlockRec block_rec(const pv_dev_cohort& C, uint64_t gblk, uint64_t grp_base, uint64_t b) {
    BlockRec r{0, 0, 0, nullptr};
    if (!CP) {
        const uint64_t loc = __ldg(C.blocks + 2 * gblk);
        r.pst = (int64_t)__ldg(C.blocks + 2 * gblk + 1);
        r.poff = loc_off(loc);
        r.plen = loc_len(loc);
        if (r.plen == (uint32_t)PV_BLOCK_CACHED) r.cache = C.cache + loc_off(loc) * C.Q;
        return r;
    }
    const uint32_t j = (uint32_t)(b & 31);
    const pv_blk_group* G = C.groups + grp_base + (b >> 5);
    const uint32_t* bt = C.btab + (gblk - j);
    const uint32_t emask = __ldg(&G->exc_mask);
    uint64_t off = __ldg(&G->off);
    int64_t st = __ldg(&G->state);
    uint32_t e = __ldg(&G->exc_base);
    for (uint32_t k = 1; k <= j; k++) {
        off += __ldg(bt + k - 1) & 0xFFFFu;
        if ((emask >> k) & 1u) { st = __ldg(C.bexc + e++); continue; }
        const int32_t code = (int32_t)(int16_t)(__ldg(bt + k) >> 16);
        const int64_t pc = st >> 1, pred = (st & 1) ? pc - (int64_t)C.Q : pc + (int64_t)C.Q;
        st = (int64_t)((uint64_t)(pred + (code >> 1)) << 1) | (int64_t)(code & 1);
    }
    r.poff = off; r.pst = st; r.plen = __ldg(bt + j) & 0xFFFFu;
    const uint32_t cmask = __ldg(&G->cache_mask);
    if ((cmask >> j) & 1u) r.cache = C.cache + (uint64_t)(__ldg(&G->cache_base) + __popc(cmask & ((1u << j) - 1u))) * C.Q;
    return r;
}
template <bool CP>
__device__ void item_block_lane(const Params& P, Item* it) {
    const BlockRec r = block_rec<CP>(P.C, it->gblk, P.C.asms[it->a].grp_base, it->bst >> P.qshift);
    it->poff = r.poff; it->plen = r.plen; it->pst = it->cst = r.pst;
    if (r.cache) { it->state = ST_CACHED; it->cptr = r.cache; }
    else if (!CP && r.plen == (uint32_t)PV_BLEN_BAD) { it->state = ST_ERR; report(P, it->w, PV_STATUS_DECODE); }
}

// The split form's work queue, at the start of the call's scratch: pv_decode_kernel zeroes it (it runs first, and the
// two kernels after it wait for it to finish); pv_emit_kernel's warps take items from `next` and list the items that
// need the general path in `heavy`; pv_heavy_kernel's CTAs take those from `hnext`.
struct WorkQueue { unsigned long long next, nheavy, hnext, pad[5]; };
constexpr uint64_t QUEUE_BYTES = 256;
constexpr unsigned HEAVY_CTAS = 148;             // pv_heavy_kernel's grid (each CTA a Q-byte block buffer in the scratch)

constexpr int DEC_THREADS = 32;            // one warp per CTA: the few decode warps of a call spread over all SMs
constexpr uint64_t DEC_WARPS = 3072;       // decode warps a split call aims for (148 SMs x ~21)
template <bool PK, bool CP>
__global__ void __launch_bounds__(DEC_THREADS, 24) pv_decode_kernel(const __grid_constant__ Params P, Item* plan, WorkQueue* q) {
    pdl_trigger();                                  // the emission kernel's CTAs may be placed now; they wait for this grid
    pdl_wait();
    if (blockIdx.x == 0 && threadIdx.x == 0) { q->next = 0; q->nheavy = 0; q->hnext = 0; }
    if (threadIdx.x >= P.dec_lanes) return;
    const uint64_t i = (uint64_t)blockIdx.x * P.dec_lanes + threadIdx.x;
    if (i >= P.total) return;
    Item* it = plan + i;
    trace_at(P, i, 0);
    if (!item_locate(P, i, it)) return;
    const pv_dev_cohort& C = P.C;
    // the item's lower-case runs are found by this lane once its decode is done (the emission kernel then copies
    // them with the item's header); the block's first run is loaded now, so that its latency overlaps the decode
    const uint32_t brun0 = C.brun ? __ldg(C.brun + it->gblk) : 0u;
    // with a checkpoint index the item's checkpoint says everything the decode needs (block validated or not, served
    // from the cache or not, its stream position); the block table is read only for the general path.
    if (C.ckpt) item_ckpt(P, it);
    else item_block_lane<CP>(P, it);
    trace_at(P, i, 1);
    if (it->state != ST_LOCATED) {
        if (it->state == ST_CACHED) item_runs_from(P, it, brun0);
        return;
    }
    item_span(P, it, false, ~0ull);              // (L2 only: any length)
    if (!PK && it->span_len)        // (evict-last: the call's output stores should not push it out before the emission reads it)
        asm volatile("cp.async.bulk.prefetch.L2.global.L2::cache_hint [%0], %1, %2;" :: "l"(C.ref + it->span_lo), "r"(it->span_len),
                     "l"(l2_evict_last()) : "memory");
    int r = DEC_ABORT;
    if (!P.force_block) {
        WindowSink sk{it->ops, it->lits, it->ox0, it->ox1, 0, 0};
        const RefView R{C.ref, C.ref_n, 0, 0, 0, PK ? C.pref : nullptr, C.pruns, C.pidx};
        trace_at(P, i, 2);
        if (it->ck != NO_CK) {                   // from its checkpoint to the item's end
            Dec<OpenStream> d;
            dec_init_ck(d, OpenStream{C.payload + it->cpos}, C.ckpt + it->ck);
            r = decode_events(d, GlobalTab{C.tabs + it->tab_off}, R, it->blen, it->ox1, sk, true);
        } else {                                 // the whole block, from its start
            Dec<GlobalStream> d;
            const uint8_t* src = C.payload + it->poff;
            dec_init(d, GlobalStream{src, src + it->plen}, it->pst);
            r = decode_events(d, GlobalTab{C.tabs + it->tab_off}, R, it->blen, it->blen, sk);
        }
        trace_at(P, i, 3);
        it->nops = (uint16_t)sk.nops; it->nlits = (uint16_t)sk.nlits;
    }
    if (r == DEC_DONE) { it->state = ST_OK; item_runs_from(P, it, brun0); }
    else if (r == DEC_ABORT) {                   // the general path decodes the block from its start: its record
        if (C.ckpt) item_block_lane<CP>(P, it);
        if (it->state == ST_LOCATED) it->state = ST_HEAVY;
    } else { it->state = ST_ERR; report(P, it->w, PV_STATUS_DECODE); }
}

// pv_emit_kernel: persistent - as many CTAs as are resident at once - and each WARP on its own takes the next decoded
// item from the queue and writes it: the item's header (with the lower-case runs its decode lane found) is copied
// into the warp's small shared slot, its ops and literal bytes are read in place from the plan, and the reference
// bytes from global memory, where the decode kernel has just warmed the item's span into L2 - no staging and no wait,
// so a warp goes from one item to the next at once, and a slot is a few hundred bytes (many warps per SM). A warp
// that finishes takes the next item: no CTA-wide barrier. Items that need the general path are listed for
// pv_heavy_kernel.
constexpr int EMIT_SLOT = ITEM_HEAD16 * 16;
template <bool PK>
__global__ void __launch_bounds__(CTA, 8) pv_emit_kernel(const __grid_constant__ Params P, const Item* plan, WorkQueue* q, uint64_t* heavy) {
    extern __shared__ uint4 smem_raw[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    pdl_trigger();                                  // pv_heavy_kernel's CTAs may be placed now; they wait for this grid
    pdl_wait();
    Item* it = (Item*)((uint8_t*)smem_raw + (size_t)warp * EMIT_SLOT);   // (the header part of an Item only)
    const pv_dev_cohort& C = P.C;
    const RefView R{C.ref, C.ref_n, 0, 0, 0, PK ? C.pref : nullptr, C.pruns, C.pidx};
    for (uint64_t round = 0; round <= P.total; round++) {      // (bounded: every round takes an item or ends)
        uint64_t item = 0;
        if (lane == 0) item = atomicAdd(&q->next, 1ull);
        item = __shfl_sync(0xffffffffu, item, 0);
        if (item >= P.total) break;
        if (lane == 0) trace_at(P, item, 4);
        const Item* pi = plan + item;
        const uint4* src = (const uint4*)pi;
        for (uint32_t k = lane; k < ITEM_HEAD16; k += 32) ((uint4*)it)[k] = __ldg(src + k);
        __syncwarp();
        const int st0 = it->state;
        if (st0 == ST_HEAVY) {
            if (lane == 0) heavy[atomicAdd(&q->nheavy, 1ull)] = item;
            __syncwarp();
            continue;
        }
        if (st0 == ST_OK || st0 == ST_CACHED) {     // (the decode kernel found the item's runs)
            if (lane == 0) trace_at(P, item, 5);
            if (st0 == ST_OK) emit_ops<true>(P, it, pi->ops, LitSrc{0, pi->lits, PK ? nullptr : C.rcref, l2_evict_first()}, R, lane);
            else emit_cached(P, it, lane);
        }
        __syncwarp();
        if (lane == 0 && st0 != ST_IDLE) trace_done(P, it, 2);
        __syncwarp();
    }
}

// pv_heavy_kernel: the items listed by pv_emit_kernel (a self copy inside the window, more ops or literals than a
// slot holds, a stream longer than a slot, or every item under PV_WIN_BLOCK_PATH), one per CTA at a time: the CTA
// decodes the block from its start into its block buffer and emits the item's range (heavy_item). Usually there are
// none, and each CTA finds the list empty and returns.
template <bool PK>
__global__ void __launch_bounds__(CTA) pv_heavy_kernel(const __grid_constant__ Params P, const Item* plan, WorkQueue* q, const uint64_t* heavy) {
    extern __shared__ uint4 smem_raw[];
    __shared__ Op hops[HOPS];
    __shared__ uint64_t h_item;
    pdl_wait();
    uint8_t* slot = (uint8_t*)smem_raw;
    Item* it = slot_item(slot);
    uint8_t* buf = P.work + (uint64_t)blockIdx.x * P.C.Q;
    const uint64_t nheavy = *(volatile unsigned long long*)&q->nheavy;
    for (uint64_t round = 0; round <= nheavy; round++) {
        if (threadIdx.x == 0) {
            const unsigned long long h = atomicAdd(&q->hnext, 1ull);
            h_item = h < nheavy ? heavy[h] : ~0ull;
        }
        __syncthreads();
        const uint64_t item = h_item;
        if (item == ~0ull) break;
        const uint4* src = (const uint4*)(plan + item);
        for (uint32_t k = threadIdx.x; k < sizeof(Item) / 16; k += CTA) ((uint4*)it)[k] = __ldg(src + k);
        __syncthreads();
        if (threadIdx.x == 0) { it->span_len = 0; it->span_lo = 0; item_runs(P, it); }   // the reference from global memory
        __syncthreads();
        heavy_item<PK, true>(P, slot, buf, hops);
        if (threadIdx.x == 0) trace_done(P, it, 2);
        __syncthreads();
    }
}

// ---------------------------------------------------------------- the checkpoint index (pv_index_build)
// A block decoded once, from its start, by one lane; at every event boundary the sink sees the decoder's state and
// writes it into the checkpoints whose offsets j S it is the last boundary at or before (pv_ckpt, packed the same way
// dec_init_ck unpacks it).
// It also counts each cell's decode cost - the events that start in it and the literal bytes decoded in it - and keeps
// the largest: the serial work of the block's costliest window item.
struct CkptSink {
    uint4* out;                  // the block's checkpoints, two uint4 each
    const uint8_t* base;         // the pooled payload's first byte
    uint32_t cs, ncell, jn;      // stride shift, checkpoints per block, the next one to write
    uint4 sa, sb;                // the last event boundary's state
    uint32_t cell, cost, worst;  // the current cell, its cost so far, the largest cost of a finished cell
    __device__ __forceinline__ void put(uint32_t j) { out[2 * j] = sa; out[2 * j + 1] = sb; }
    __device__ __forceinline__ void at(const Dec<GlobalStream>& d) {
        const uint32_t cj = d.o >> cs;
        if (cj != cell) { worst = cost > worst ? cost : worst; cost = 0; cell = cj; }
        cost++;
        while (jn < ncell && (jn << cs) < d.o) put(jn++);
        const uint64_t c[4] = {d.c0 + (uint64_t)PV_CKPT_BIAS, d.c1 + (uint64_t)PV_CKPT_BIAS, d.c2 + (uint64_t)PV_CKPT_BIAS,
                               d.c3 + (uint64_t)PV_CKPT_BIAS};
        sa.x = d.x | (d.pk << 24) | ((uint32_t)(d.nc - 1) << 27);
        const uint64_t pos = (uint64_t)(d.st.p - base);
        sa.y = (uint32_t)pos;
        sa.z = (uint32_t)c[0]; sa.w = (uint32_t)c[1]; sb.x = (uint32_t)c[2]; sb.y = (uint32_t)c[3];
        sb.z = ((uint32_t)(c[0] >> 32) & 0x7Fu) | (d.d0 << 7) | ((((uint32_t)(c[1] >> 32) & 0x7Fu) | (d.d1 << 7)) << 8) |
               ((((uint32_t)(c[2] >> 32) & 0x7Fu) | (d.d2 << 7)) << 16) | ((((uint32_t)(c[3] >> 32) & 0x7Fu) | (d.d3 << 7)) << 24);
        sb.w = d.o | (uint32_t)(((pos >> 32) & 0xFFu) << 24);
    }
    __device__ bool more() const { return true; }
    __device__ bool lit(uint32_t, uint8_t) { cost++; return true; }
    __device__ bool op(uint32_t, uint64_t, uint32_t, uint32_t) { return true; }
    __device__ uint32_t costliest() const { return cost > worst ? cost : worst; }
};

template <bool PK, bool CP>
__global__ void __launch_bounds__(128) pv_index_kernel(const pv_dev_cohort C, uint64_t nblk, uint32_t cs, uint32_t qs, uint4* out,
                                                       unsigned long long* nbad, uint32_t* brun, uint16_t* cost) {
    const uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= nblk) return;
    int64_t lo = 0, hi = C.nasm;                    // the assembly: the last one whose first block is at or before i
    while (hi - lo > 1) { const int64_t m = (lo + hi) >> 1; if (__ldg(&C.asms[m].blk_base) <= i) lo = m; else hi = m; }
    const pv_asm_rec& R = C.asms[lo];
    const uint64_t b = i - __ldg(&R.blk_base), nbases = __ldg(&R.nbases), bst = b << qs;
    const uint32_t blen = (uint32_t)(nbases - bst < (1ull << qs) ? nbases - bst : (1ull << qs));
    const uint32_t ncell = 1u << (qs - cs);
    uint4* o = out + 2 * (i << (qs - cs));
    if (brun) {                                     // the block's first lower-case run: the first to end after bst
        const uint64_t* low = C.low + 2 * __ldg(&R.low_base);
        uint64_t lo = 0, hi = __ldg(&R.low_cnt);
        while (lo < hi) { const uint64_t m = (lo + hi) >> 1; if (__ldg(low + 2 * m + 1) <= bst) lo = m + 1; else hi = m; }
        brun[i] = (uint32_t)lo;
    }
    const BlockRec r = block_rec<CP>(C, i, __ldg(&R.grp_base), b);
    if (r.cache) {                                  // served from the block cache: its row, for every cell
        const uint32_t slot = (uint32_t)((uint64_t)(r.cache - C.cache) >> qs);
        for (uint32_t j = 0; j < ncell; j++) { o[2 * j] = make_uint4(0, slot, 0, 0); o[2 * j + 1] = make_uint4(0, 0, 0, PV_CKPT_CACHED << 16); }
        if (cost) cost[i] = 0;
        return;
    }
    int res = DEC_ERR;
    uint32_t worst = 0;
    if (CP || r.plen != (uint32_t)PV_BLEN_BAD) {
        const uint8_t* src = C.payload + r.poff;
        CkptSink sk{o, C.payload, cs, ncell, 0, make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0), 0, 0, 0};
        Dec<GlobalStream> d;
        dec_init(d, GlobalStream{src, src + r.plen}, r.pst);
        const RefView V{C.ref, C.ref_n, 0, 0, 0, PK ? C.pref : nullptr, C.pruns, C.pidx};
        res = decode_events(d, GlobalTab{C.tabs + __ldg(&R.tab_off)}, V, blen, blen, sk);
        if (res == DEC_DONE) while (sk.jn < ncell) sk.put(sk.jn++);   // the last boundary's state for the rest
        worst = sk.costliest();
    }
    if (cost) cost[i] = (uint16_t)(res == DEC_DONE ? (worst < 0xFFFFu ? worst : 0xFFFFu) : 0u);
    if (res != DEC_DONE) {
        for (uint32_t j = 0; j < ncell; j++) { o[2 * j] = make_uint4(0, 0, 0, 0); o[2 * j + 1] = make_uint4(0, 0, 0, PV_CKPT_BAD << 16); }
        if (nbad) atomicAdd(nbad, 1ull);
    }
}

// ---------------------------------------------------------------- sample() coordinates
// The arithmetic between sample()'s draws and its window decode (panvram/cohort.py:177-189, 193-194): u uniform over all valid
// starts -> contig k = searchsorted(cum, u, right=True), pos = u - (cum[k] - v[k]), assembly and base-stream start,
// strand from the rand() draw. One warp per window: a 32-way search (each level one load per lane and a ballot), so
// 3 dependent loads cover 32,768 contigs.
// sample()'s draws made in the coordinate kernel, as torch's CUDA kernels make them for torch.randint(0, total, (n,)) and
// torch.rand(n) (ATen/native/cuda/DistributionTemplates.h: a grid-stride loop of `threads` threads, thread t's Philox
// state curand_init(seed, t, offset); each curand4 call gives `unroll` values, element li taking value
// (li mod threads x unroll) / threads of call li / (threads x unroll); randint keeps 64 bits (two words) per value for
// a range of 2^28 or more and reduces them mod the range; rand maps curand_uniform's (0, 1] to [0, 1) by sending 1 to
// 0). rng (device) holds the generator's seed and offset; the launch's last CTA advances the offset by what torch's two
// calls would, so a captured graph replays the generator's stream call after call.
struct TorchDraws {
    pv_philox* rng;             // the generator state on the device (advanced by the launch), or NULL
    uint64_t total, threads, inc_int, inc_all;
    int64_t* u_out; float* r_out;   // the draws themselves (for tests), or NULL
    uint64_t seed, offset;      // the generator state as arguments (rng NULL, draw 1)
    int draw;                   // make the draws (else they come from u / r)
};
struct CoordParams {
    const int64_t *cum, *v, *casm, *cboff, *clocal, *u;
    const float* r;
    int64_t nctg, n;
    float p;
    int rc_mode;
    int64_t *asm_out, *start_out, *coords;
    uint8_t* rc_out;
    int32_t* status;
    TorchDraws D;
};
constexpr int COORD_WARPS = 8;

__device__ __noinline__ int64_t torch_randint(uint64_t seed, uint64_t off, uint64_t threads, uint64_t total, uint64_t li) {
    const bool wide = total >= (1ull << 28);
    const uint64_t per = threads * (wide ? 2 : 4), pass = li / per, rem = li - pass * per, ii = rem / threads;
    curandStatePhilox4_32_10_t st;
    curand_init(seed, rem - ii * threads, off, &st);
    uint4 v = curand4(&st);
    for (uint64_t k = 0; k < pass; k++) v = curand4(&st);
    const uint64_t val = wide ? (ii == 0 ? ((uint64_t)v.x << 32 | v.y) : ((uint64_t)v.z << 32 | v.w))
                              : (uint64_t)(ii == 0 ? v.x : ii == 1 ? v.y : ii == 2 ? v.z : v.w);
    return (int64_t)(val % total);
}
__device__ __noinline__ float torch_rand(uint64_t seed, uint64_t off, uint64_t threads, uint64_t li) {
    const uint64_t per = threads * 4, pass = li / per, rem = li - pass * per, ii = rem / threads;
    curandStatePhilox4_32_10_t st;
    curand_init(seed, rem - ii * threads, off, &st);
    float4 f = curand_uniform4(&st);
    for (uint64_t k = 0; k < pass; k++) f = curand_uniform4(&st);
    const float x = ii == 0 ? f.x : ii == 1 ? f.y : ii == 2 ? f.z : f.w;
    return x == 1.0f ? 0.0f : x;
}

__global__ void __launch_bounds__(COORD_WARPS * 32) pv_sample_coords_kernel(const CoordParams P) {
    pdl_trigger();                                  // the window kernel's CTAs may be placed now; they wait for this grid
    pdl_wait();
    const int lane = threadIdx.x & 31;
    const int64_t w = (int64_t)blockIdx.x * COORD_WARPS + (threadIdx.x >> 5);
    if (w == 0 && lane == 0 && P.status) *P.status = 0;
    if (w < P.n) {                                      // (warp-uniform)
        int64_t u = 0;
        float r = 0.0f;
        if (P.D.draw) {
            if (lane == 0) {
                const uint64_t seed = P.D.rng ? __ldcg(&P.D.rng->seed) : P.D.seed, off = P.D.rng ? __ldcg(&P.D.rng->offset) : P.D.offset;
                u = torch_randint(seed, off, P.D.threads, P.D.total, (uint64_t)w);
                if (P.rc_mode == 2) r = torch_rand(seed, off + P.D.inc_int, P.D.threads, (uint64_t)w);
                if (P.D.u_out) P.D.u_out[w] = u;
                if (P.D.r_out && P.rc_mode == 2) P.D.r_out[w] = r;
            }
            u = __shfl_sync(0xffffffffu, u, 0);
        } else {
            u = P.u[w];
            if (P.rc_mode == 2 && lane == 0) r = P.r[w];
        }
        int64_t lo = 0, hi = P.nctg;                    // the answer (first k with cum[k] > u) lies in [lo, hi)
        while (hi - lo > 1) {
            const int64_t step = (hi - lo + 31) / 32;
            const int64_t idx = lo + (int64_t)(lane + 1) * step - 1;   // lane 31's probe is at or past hi - 1
            const bool above = idx >= hi - 1 || __ldg(P.cum + idx) > u;
            const int f = __ffs(__ballot_sync(0xffffffffu, above)) - 1;
            lo += (int64_t)f * step;
            hi = min(hi, lo + step);
        }
        if (lane == 0) {
            const int64_t k = lo, pos = u - (__ldg(P.cum + k) - __ldg(P.v + k)), a = __ldg(P.casm + k);
            const uint8_t s = P.rc_mode == 1 ? 1 : P.rc_mode == 2 ? (uint8_t)(r < P.p) : 0;
            P.asm_out[w] = a;
            P.start_out[w] = __ldg(P.cboff + k) + pos;
            if (P.rc_out) P.rc_out[w] = s;
            if (P.coords) {
                int64_t* c = P.coords + 4 * w;
                c[0] = a; c[1] = __ldg(P.clocal + k); c[2] = pos; c[3] = s;
            }
        }
    }
    if (P.D.rng) {                                      // every CTA has read the offset: the last one advances it
        __syncthreads();
        if (threadIdx.x == 0) {
            __threadfence();
            if (atomicAdd(&P.D.rng->arrived, 1u) == gridDim.x - 1) {
                P.D.rng->offset += P.D.inc_all;
                P.D.rng->arrived = 0;
                __threadfence();
            }
        }
    }
}

// window coordinates read from pinned host memory through its mapped address (pv_coords_from_host)
__global__ void __launch_bounds__(256) pv_coords_from_host_kernel(const int64_t* a, const int64_t* s, const uint8_t* r, int64_t n,
                                                                  int64_t* ad, int64_t* sd, uint8_t* rd) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        ad[i] = a[i];
        sd[i] = s[i];
        if (r) rd[i] = r[i];
    }
}
// the status word stored into pinned host memory by one thread (pv_status_to_host): no copy engine involved
__global__ void pv_status_to_host_kernel(const int32_t* s, int32_t* h) {
    *(volatile int32_t*)h = *(const volatile int32_t*)s;
    __threadfence_system();
}

}  // namespace

namespace pvb { thread_local char g_cuda_err[256]; }   // pv_kernels_last_error (also set by pv_fasta.cu's launchers)
using pvb::g_cuda_err;

extern "C" {

const char* pv_kernels_last_error(void) { return g_cuda_err; }

int pv_windows_launches(int64_t n, int64_t W) { return (n > 0 && W > 0) ? 3 : 0; }   // (at most: 1 when fused)

int pv_coords_from_host(const int64_t* asm_host, const int64_t* start_host, const uint8_t* rc_host, int64_t n, int64_t* asm_index,
                        int64_t* start, uint8_t* rc, void* stream) {
    if (n < 0 || (n > 0 && (!asm_host || !start_host || !asm_index || !start || (rc_host && !rc)))) {
        snprintf(g_cuda_err, sizeof g_cuda_err, "pv_coords_from_host: arguments");
        return PV_EARG;
    }
    if (n == 0) return PV_OK;
    const int64_t *a = nullptr, *s = nullptr;
    const uint8_t* r = nullptr;
    if (cudaHostGetDevicePointer((void**)&a, (void*)asm_host, 0) != cudaSuccess || !a ||
        cudaHostGetDevicePointer((void**)&s, (void*)start_host, 0) != cudaSuccess || !s ||
        (rc_host && (cudaHostGetDevicePointer((void**)&r, (void*)rc_host, 0) != cudaSuccess || !r))) {
        cudaGetLastError();
        snprintf(g_cuda_err, sizeof g_cuda_err, "pv_coords_from_host: the host arrays must be pinned (cudaHostAlloc) memory");
        return PV_EARG;
    }
    const int64_t grid = std::min<int64_t>((n + 255) / 256, 148 * 4);
    pv_coords_from_host_kernel<<<(unsigned)grid, 256, 0, (cudaStream_t)stream>>>(a, s, r, n, asm_index, start, rc);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) { snprintf(g_cuda_err, sizeof g_cuda_err, "%s", cudaGetErrorString(e)); return PV_ECUDA; }
    return PV_OK;
}

int pv_status_to_host(const int32_t* status, int32_t* host_word, void* stream) {
    int32_t* d = nullptr;
    if (!status || !host_word || cudaHostGetDevicePointer((void**)&d, host_word, 0) != cudaSuccess || !d) {
        cudaGetLastError();
        snprintf(g_cuda_err, sizeof g_cuda_err, "pv_status_to_host: the host word must be pinned (cudaHostAlloc) memory");
        return PV_EARG;
    }
    pv_status_to_host_kernel<<<1, 1, 0, (cudaStream_t)stream>>>(status, d);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) { snprintf(g_cuda_err, sizeof g_cuda_err, "%s", cudaGetErrorString(e)); return PV_ECUDA; }
    return PV_OK;
}

// an item's cell: the checkpoint stride of a cohort with an index, else the block (items = (window, cell touched))
static uint32_t cell_of(const pv_dev_cohort* c) { return c->ckpt ? 1u << c->ckpt_shift : c->Q; }
static uint64_t grid_of(uint32_t cell, int64_t n, int64_t W, uint64_t* total, uint64_t* bpw) {
    *bpw = ((uint64_t)W + cell - 1) / cell + 1;
    *total = (uint64_t)n * *bpw;
    return (*total + WARPS - 1) / WARPS;
}

// scratch: the plan (one Item per item, the split pipeline's decode results), then a Q-byte general-path buffer per CTA
// the fused kernel below this many items (n x blocks per window), the split form from it: where they cross, measured
// on B200 with W = 8,192 (q4k: equal at 4,608 items, fused 20 % faster at 3,072; q16k: fused 22 % faster at 2,048,
// split 6 % faster at 4,096; a q16k item decodes a 4x longer stream, so the split form pays off sooner)
static uint64_t split_min_items(uint32_t cell) { return cell >= 16384 ? 3072 : 4608; }
// the form a call of `total` items takes (true: fused) and, for the split form, its items per decode warp: enough that
// the call runs about DEC_WARPS decode warps (~21 per SM; fewer chains per warp diverge less, and beyond that many
// warps the SMs' issue slots are full anyway; measured, 1.5 K-49 K items), at most 32
static bool form_of(uint32_t cell, uint64_t total, uint32_t flags, uint32_t* lanes) {
    const uint32_t k = (flags >> PV_WIN_DEC_LANES_SHIFT) & 63u;
    *lanes = k ? k : (uint32_t)std::min<uint64_t>(32, std::max<uint64_t>(1, (total + DEC_WARPS - 1) / DEC_WARPS));
    return (flags & PV_WIN_FUSED) ? true : (flags & PV_WIN_SPLIT) ? false : total < split_min_items(cell);
}
static uint64_t plan_bytes(uint64_t total) { return (total * sizeof(Item) + 255) & ~255ull; }
// A call's scratch. The split form: its work queue, the plan (one Item per item), the list of items for the general
// path, and pv_heavy_kernel's Q-byte block buffers. The fused form: a Q-byte block buffer per CTA. Sized for either.
static uint64_t split_scratch(uint64_t total, uint32_t Q) {
    return QUEUE_BYTES + plan_bytes(total) + ((8 * total + 255) & ~255ull) + (uint64_t)HEAVY_CTAS * Q;
}
static uint64_t work_need(uint64_t total, uint64_t grid, uint32_t Q) { return std::max<uint64_t>(split_scratch(total, Q), grid * Q); }
size_t pv_windows_work_bytes(const pv_dev_cohort* cohort, int64_t n, int64_t W) {
    if (n <= 0 || W <= 0) return 0;
    uint64_t total, bpw;
    const uint64_t grid = grid_of(cell_of(cohort), n, W, &total, &bpw);
    return (size_t)work_need(total, grid, cohort->Q);
}

int pv_windows(const pv_dev_cohort* cohort, const int64_t* asm_index, const int64_t* start, int64_t n, int64_t W, const uint8_t* rc,
               int tokens, int apply_case, uint8_t* out, int32_t* status, void* work, size_t work_bytes, void* stream) {
    return pv_windows_ex(cohort, asm_index, start, n, W, rc, tokens, apply_case, 0u, out, status, nullptr, work, work_bytes, stream);
}

}  // extern "C"

// a launch with programmatic stream serialisation allowed (the kernel waits in pdl_wait for the one before it)
template <typename... K, typename... A>
static cudaError_t launch_pdl(void (*k)(K...), unsigned grid, unsigned block, size_t smem, cudaStream_t st, A&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid); cfg.blockDim = dim3(block); cfg.dynamicSmemBytes = smem; cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at; cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, k, std::forward<A>(args)...);
}

// kernel launches per resident form (packed reference / compact block table), each with its dynamic shared memory
// attribute set once per device and size
static cudaError_t smem_attr(const void* fn, int slot, size_t smem) {
    static size_t set[12][64] = {{0}};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && smem <= set[slot][dev]) return cudaSuccess;
    const cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e == cudaSuccess && dev >= 0 && dev < 64) set[slot][dev] = smem;
    return e;
}
template <bool PK, bool CP>
static cudaError_t fused_form(uint64_t grid, size_t smem, cudaStream_t st, const Params& P) {
    const cudaError_t e = smem_attr((const void*)pv_windows_kernel<PK, CP>, (PK ? 1 : 0) | (CP ? 2 : 0), smem);
    if (e != cudaSuccess) return e;
    return launch_pdl(pv_windows_kernel<PK, CP>, (unsigned)grid, CTA, smem, st, P);
}
// CTAs of a kernel resident at once on the current device (its SM count x what fits on an SM), cached per kernel and size
struct ResidentMemo { const void* fn; size_t smem; int dev; unsigned n; };
static unsigned resident_ctas(const void* fn, int block, size_t smem) {
    static thread_local ResidentMemo memo[16];
    static thread_local int next = 0;
    int dev = 0;
    cudaGetDevice(&dev);
    for (int i = 0; i < 16; i++)
        if (memo[i].fn == fn && memo[i].smem == smem && memo[i].dev == dev) return memo[i].n;
    int sms = 0, per = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, fn, block, smem) != cudaSuccess || per < 1) {
        cudaGetLastError();
        return 148;
    }
    const unsigned n = (unsigned)(sms * per);
    memo[next] = ResidentMemo{fn, smem, dev, n};
    next = (next + 1) % 16;
    return n;
}
// decode kernel, then the persistent emission kernel (no more CTAs than are resident at once, nor than its items need),
// then the general-path kernel
template <bool PK, bool CP>
static cudaError_t split_form(uint64_t total, size_t smem_e, cudaStream_t st, const Params& P, const Params& PE, const Params& PH, Item* plan,
                              WorkQueue* q, uint64_t* heavy) {
    cudaError_t e = smem_attr((const void*)pv_emit_kernel<PK>, 4 + (PK ? 1 : 0), smem_e);
    if (e != cudaSuccess) return e;
    e = launch_pdl(pv_decode_kernel<PK, CP>, (unsigned)((total + P.dec_lanes - 1) / P.dec_lanes), DEC_THREADS, 0, st, P, plan, q);
    if (e != cudaSuccess) return e;
    const uint64_t want = (total + WARPS - 1) / WARPS;
    const uint64_t resident = resident_ctas((const void*)pv_emit_kernel<PK>, CTA, smem_e);
    const unsigned grid = (unsigned)(want < resident ? want : resident);
    e = launch_pdl(pv_emit_kernel<PK>, grid, CTA, smem_e, st, PE, (const Item*)plan, q, heavy);
    if (e != cudaSuccess) return e;
    return launch_pdl(pv_heavy_kernel<PK>, HEAVY_CTAS, CTA, sizeof(Item), st, PH, (const Item*)plan, q, (const uint64_t*)heavy);
}
static cudaError_t launch_fused(int form, uint64_t grid, size_t smem, cudaStream_t st, const Params& P) {
    switch (form) {
    case 0: return fused_form<false, false>(grid, smem, st, P);
    case 1: return fused_form<true, false>(grid, smem, st, P);
    case 2: return fused_form<false, true>(grid, smem, st, P);
    default: return fused_form<true, true>(grid, smem, st, P);
    }
}
static cudaError_t launch_split(int form, uint64_t total, size_t smem_e, cudaStream_t st, const Params& P, const Params& PE,
                                const Params& PH, Item* plan, WorkQueue* q, uint64_t* heavy) {
    switch (form) {
    case 0: return split_form<false, false>(total, smem_e, st, P, PE, PH, plan, q, heavy);
    case 1: return split_form<true, false>(total, smem_e, st, P, PE, PH, plan, q, heavy);
    case 2: return split_form<false, true>(total, smem_e, st, P, PE, PH, plan, q, heavy);
    default: return split_form<true, true>(total, smem_e, st, P, PE, PH, plan, q, heavy);
    }
}

static int launch_windows(const pv_dev_cohort* cohort, const int64_t* asm_index, const int64_t* start, int64_t n, int64_t W,
                          const uint8_t* rc, int tokens, int apply_case, uint32_t flags, uint8_t* out, int64_t* out64,
                          const int64_t* ids, int32_t* status, uint8_t* wstatus, void* work, size_t work_bytes, void* stream,
                          uint64_t* trace = nullptr, size_t trace_records = 0) {
    const uint32_t Q = cohort->Q;
    if ((cohort->packed && (!cohort->pref || !cohort->pruns || !cohort->pidx)) ||
        (cohort->compact && (!cohort->groups || !cohort->btab || !cohort->bexc)) || (!cohort->packed && !cohort->ref) ||
        (!cohort->compact && !cohort->blocks)) {
        snprintf(g_cuda_err, sizeof g_cuda_err, "cohort: the arrays of its resident form are missing");
        return PV_EARG;
    }
    if (!(Q == 1024 || Q == 2048 || Q == 4096 || Q == 16384)) { snprintf(g_cuda_err, sizeof g_cuda_err, "block size"); return PV_EARG; }
    if (W < 0 || W >= (1ll << 31)) { snprintf(g_cuda_err, sizeof g_cuda_err, "W"); return PV_EARG; }
    if (n < 0) { snprintf(g_cuda_err, sizeof g_cuda_err, "n"); return PV_EARG; }
    if (cohort->tab_max > PV_TAB_MAX_BYTES || cohort->tab_max % 16) { snprintf(g_cuda_err, sizeof g_cuda_err, "decode table size"); return PV_EARG; }
    uint32_t qshift = 0;
    while ((1u << qshift) < Q) qshift++;
    if (cohort->ckpt && (cohort->ckpt_shift < 8 || cohort->ckpt_shift > qshift)) {
        snprintf(g_cuda_err, sizeof g_cuda_err, "checkpoint stride: 256 to Q");
        return PV_EARG;
    }
    if (n == 0 || W == 0) return PV_OK;
    const uint32_t cell = cell_of(cohort);
    Params P;
    P.C = *cohort; P.wasm = asm_index; P.wstart = start; P.rc = rc; P.out = out; P.status = status; P.wstatus = wstatus;
    P.out64 = out64;
    for (int k = 0; k < 5; k++) P.ids[k] = ids ? ids[k] : 0;
    P.n = (uint64_t)n; P.W = (uint64_t)W;
    if ((uint64_t)n > (1ull << 62) / (((uint64_t)W + cell - 1) / cell + 1)) { snprintf(g_cuda_err, sizeof g_cuda_err, "too many blocks in one call"); return PV_EARG; }
    const uint64_t grid = grid_of(cell, n, W, &P.total, &P.bpw);
    if (grid >= (1ull << 31)) { snprintf(g_cuda_err, sizeof g_cuda_err, "too many blocks in one call"); return PV_EARG; }
    // the fused kernel for calls of few items (each warp's one chain then overlaps the others' well); the decode +
    // emission pair beyond, where several chains per decode warp amortise the decode
    if (((flags >> PV_WIN_DEC_LANES_SHIFT) & 63u) > 32) { snprintf(g_cuda_err, sizeof g_cuda_err, "decode lanes per warp: 1 to 32"); return PV_EARG; }
    const bool fused = form_of(cell, P.total, flags, &P.dec_lanes);
    const uint64_t need = work_need(P.total, grid, Q);
    if (!work || work_bytes < need || ((uintptr_t)work & 15)) {
        snprintf(g_cuda_err, sizeof g_cuda_err, "work buffer: %llu bytes needed, 16-byte aligned", (unsigned long long)need);
        return PV_EARG;
    }
    if (trace && (trace_records < P.total || ((uintptr_t)trace & 7))) {
        snprintf(g_cuda_err, sizeof g_cuda_err, "trace: %llu records of 8 words needed", (unsigned long long)P.total);
        return PV_EARG;
    }
    P.trace = trace;
    // the split form's scratch: queue | plan | general-path list | block buffers; the fused form's: block buffers
    WorkQueue* q = (WorkQueue*)work;
    Item* plan = (Item*)((uint8_t*)work + QUEUE_BYTES);
    uint64_t* heavy = (uint64_t*)((uint8_t*)plan + plan_bytes(P.total));
    uint8_t* hbuf = (uint8_t*)heavy + ((8 * P.total + 255) & ~255ull);
    P.work = (uint8_t*)work;
    P.tokens = tokens; P.apply_case = apply_case; P.force_block = (flags & PV_WIN_BLOCK_PATH) ? 1 : 0;
    P.test_wait = (flags & PV_WIN_TEST_WAIT) ? 1 : 0;
    P.qshift = qshift;
    P.cshift = cohort->ckpt ? cohort->ckpt_shift : qshift;
    P.tab_area = (uint32_t)((cohort->tab_max + 15) & ~15ull);
    P.pay_cap = ((Q / 32 + 32 < 160 ? 160 : Q / 32 + 32) + 15) & ~15u;
    P.narrow = W < (int64_t)Q;
    // a slot's reference span: an item's range is at most min(W, Q) bases; from checkpoints it is about one stride,
    // so the slot holds two strides (a longer item reads what does not fit from global memory)
    uint64_t span = P.narrow ? (uint64_t)W : Q;
    if (cohort->ckpt && span > 2ull * cell) span = 2ull * cell;
    P.span_cap = (uint32_t)((span + 2 * SPAN_MARGIN + 64 + 15) & ~15ull);
    P.slot_bytes = (uint32_t)sizeof(Item) + P.tab_area + P.pay_cap + P.span_cap;
    const size_t smem = (size_t)WARPS * P.slot_bytes;
    // the emission kernel's slot: an item's header only (its ops and literal bytes are read in place, the reference
    // from global memory); pv_heavy_kernel's: a whole Item, no span (it reads the reference from global memory)
    Params PE = P;
    PE.pay_cap = 0;
    PE.tab_area = 0;
    PE.span_cap = 0;
    PE.slot_bytes = (uint32_t)sizeof(Item);
    const size_t smem_e = (size_t)WARPS * EMIT_SLOT;
    Params PH = PE;                                 // pv_heavy_kernel: its CTAs' block buffers after the list
    PH.work = hbuf;
    const int form = (cohort->packed ? 1 : 0) | (cohort->compact ? 2 : 0);
    const cudaError_t le = fused ? launch_fused(form, grid, smem, (cudaStream_t)stream, P)
                                 : launch_split(form, P.total, smem_e, (cudaStream_t)stream, P, PE, PH, plan, q, heavy);
    if (le != cudaSuccess) { snprintf(g_cuda_err, sizeof g_cuda_err, "%s", cudaGetErrorString(le)); return PV_ECUDA; }
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) { snprintf(g_cuda_err, sizeof g_cuda_err, "%s", cudaGetErrorString(e)); return PV_ECUDA; }
    return PV_OK;
}

extern "C" {

int pv_windows_form(uint32_t cell, int64_t n, int64_t W, uint32_t flags, int* launches, uint32_t* dec_lanes) {
    *launches = 0; *dec_lanes = 0;
    if (cell < 256 || cell > 16384 || (cell & (cell - 1)) || n < 0 || W < 0 || ((flags >> PV_WIN_DEC_LANES_SHIFT) & 63u) > 32) {
        snprintf(g_cuda_err, sizeof g_cuda_err, "pv_windows_form: arguments");
        return PV_EARG;
    }
    if (n == 0 || W == 0) return PV_OK;
    const uint64_t total = (uint64_t)n * (((uint64_t)W + cell - 1) / cell + 1);
    uint32_t lanes;
    const bool fused = form_of(cell, total, flags, &lanes);
    *launches = fused ? 1 : 3;
    *dec_lanes = fused ? 0 : lanes;
    return PV_OK;
}

int pv_windows_ex(const pv_dev_cohort* cohort, const int64_t* asm_index, const int64_t* start, int64_t n, int64_t W, const uint8_t* rc,
                  int tokens, int apply_case, uint32_t flags, uint8_t* out, int32_t* status, uint8_t* wstatus, void* work,
                  size_t work_bytes, void* stream) {
    return launch_windows(cohort, asm_index, start, n, W, rc, tokens, apply_case, flags, out, nullptr, nullptr, status, wstatus,
                          work, work_bytes, stream);
}

size_t pv_windows_items(const pv_dev_cohort* cohort, int64_t n, int64_t W) {
    if (!cohort || n <= 0 || W <= 0) return 0;
    uint64_t total, bpw;
    grid_of(cell_of(cohort), n, W, &total, &bpw);
    return (size_t)total;
}

int pv_windows_trace(const pv_dev_cohort* cohort, const int64_t* asm_index, const int64_t* start, int64_t n, int64_t W, const uint8_t* rc,
                     int tokens, int apply_case, uint32_t flags, uint8_t* out, int32_t* status, void* work, size_t work_bytes,
                     uint64_t* trace, size_t trace_records, void* stream) {
    if (!trace) { snprintf(g_cuda_err, sizeof g_cuda_err, "pv_windows_trace: the trace array"); return PV_EARG; }
    return launch_windows(cohort, asm_index, start, n, W, rc, tokens, apply_case, flags, out, nullptr, nullptr, status, nullptr,
                          work, work_bytes, stream, trace, trace_records);
}

int pv_windows_ids(const pv_dev_cohort* cohort, const int64_t* asm_index, const int64_t* start, int64_t n, int64_t W, const uint8_t* rc,
                   const int64_t* ids, int64_t* out, int32_t* status, void* work, size_t work_bytes, void* stream) {
    if (!ids) { snprintf(g_cuda_err, sizeof g_cuda_err, "pv_windows_ids: the five token ids"); return PV_EARG; }
    if (n > 0 && W > 0 && ((uintptr_t)out & 15)) { snprintf(g_cuda_err, sizeof g_cuda_err, "pv_windows_ids: out must be 16-byte aligned"); return PV_EARG; }
    return launch_windows(cohort, asm_index, start, n, W, rc, 1, 0, 0u, nullptr, out, ids, status, nullptr, work, work_bytes, stream);
}

int pv_sample_coords(const int64_t* cum, const int64_t* valid, const int64_t* ctg_asm, const int64_t* ctg_boff,
                     const int64_t* ctg_local, int64_t nctg, const int64_t* u, const float* r, float p, int rc_mode, int64_t n,
                     int64_t* asm_index, int64_t* start, uint8_t* rc, int64_t* coords, int32_t* status, void* stream) {
    if (n < 0 || n >= (1ll << 40) || nctg <= 0 || rc_mode < 0 || rc_mode > 2) {
        snprintf(g_cuda_err, sizeof g_cuda_err, "pv_sample_coords: n, contig count or rc_mode");
        return PV_EARG;
    }
    if (n == 0 && !status) return PV_OK;
    if (n > 0 && (!cum || !valid || !ctg_asm || !ctg_boff || !u || !asm_index || !start || (rc_mode == 2 && !r) || (rc_mode != 0 && !rc) ||
                  (coords && !ctg_local))) {
        snprintf(g_cuda_err, sizeof g_cuda_err, "pv_sample_coords: a required pointer is NULL");
        return PV_EARG;
    }
    CoordParams P{cum, valid, ctg_asm, ctg_boff, ctg_local, u, r, nctg, n, p, rc_mode, asm_index, start, coords, rc, status, TorchDraws{}};
    P.D.draw = 0;
    const int64_t grid = n > 0 ? (n + COORD_WARPS - 1) / COORD_WARPS : 1;
    const cudaError_t le = launch_pdl(pv_sample_coords_kernel, (unsigned)grid, COORD_WARPS * 32, 0, (cudaStream_t)stream, P);
    if (le != cudaSuccess) { snprintf(g_cuda_err, sizeof g_cuda_err, "%s", cudaGetErrorString(le)); return PV_ECUDA; }
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) { snprintf(g_cuda_err, sizeof g_cuda_err, "%s", cudaGetErrorString(e)); return PV_ECUDA; }
    return PV_OK;
}

int pv_torch_draw_geometry(int64_t n, uint64_t total, int rc_mode, int sm_count, int threads_per_sm, uint64_t* threads,
                           uint64_t* inc_int, uint64_t* inc_all) {
    *threads = *inc_int = *inc_all = 0;
    if (n < 0 || n >= (1ll << 31) || total == 0 || rc_mode < 0 || rc_mode > 2 || sm_count <= 0 || threads_per_sm < 256) {
        snprintf(g_cuda_err, sizeof g_cuda_err, "pv_torch_draw_geometry: arguments");
        return PV_EARG;
    }
    if (n == 0) return PV_OK;                           // torch draws nothing and leaves the offset
    const uint64_t grid = std::min<uint64_t>((uint64_t)sm_count * (uint64_t)(threads_per_sm / 256), ((uint64_t)n + 255) / 256);
    *threads = 256 * grid;
    const uint64_t un = total >= (1ull << 28) ? 2 : 4;
    *inc_int = (((uint64_t)n - 1) / (*threads * un) + 1) * 4;
    *inc_all = *inc_int + (rc_mode == 2 ? (((uint64_t)n - 1) / (*threads * 4) + 1) * 4 : 0);
    return PV_OK;
}

int pv_sample_draw_coords(const int64_t* cum, const int64_t* valid, const int64_t* ctg_asm, const int64_t* ctg_boff,
                          const int64_t* ctg_local, int64_t nctg, uint64_t total, pv_philox* rng, uint64_t seed, uint64_t offset,
                          float p, int rc_mode, int64_t n, int64_t* asm_index, int64_t* start, uint8_t* rc, int64_t* coords,
                          int32_t* status, int64_t* u_out, float* r_out, void* stream) {
    if (n < 0 || n >= (1ll << 31) || nctg <= 0 || rc_mode < 0 || rc_mode > 2 || total == 0) {
        snprintf(g_cuda_err, sizeof g_cuda_err, "pv_sample_draw_coords: n, contig count, rc_mode, total or rng");
        return PV_EARG;
    }
    if (n > 0 && (!cum || !valid || !ctg_asm || !ctg_boff || !asm_index || !start || (rc_mode != 0 && !rc) || (coords && !ctg_local))) {
        snprintf(g_cuda_err, sizeof g_cuda_err, "pv_sample_draw_coords: a required pointer is NULL");
        return PV_EARG;
    }
    int dev = 0, sms = 0, tps = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&tps, cudaDevAttrMaxThreadsPerMultiProcessor, dev) != cudaSuccess) {
        snprintf(g_cuda_err, sizeof g_cuda_err, "pv_sample_draw_coords: device attributes");
        return PV_ECUDA;
    }
    TorchDraws D{rng, total, 0, 0, 0, u_out, r_out, seed, offset, 1};
    if (pv_torch_draw_geometry(n, total, rc_mode, sms, tps, &D.threads, &D.inc_int, &D.inc_all) != PV_OK) return PV_EARG;
    CoordParams P{cum, valid, ctg_asm, ctg_boff, ctg_local, nullptr, nullptr, nctg, n, p, rc_mode, asm_index, start, coords, rc, status, D};
    const int64_t grid = n > 0 ? (n + COORD_WARPS - 1) / COORD_WARPS : 1;
    const cudaError_t le = launch_pdl(pv_sample_coords_kernel, (unsigned)grid, COORD_WARPS * 32, 0, (cudaStream_t)stream, P);
    if (le != cudaSuccess) { snprintf(g_cuda_err, sizeof g_cuda_err, "%s", cudaGetErrorString(le)); return PV_ECUDA; }
    return PV_OK;
}

}  // extern "C"

// ---------------------------------------------------------------- the reverse-complement reference (pv_rc_reference)
__global__ void __launch_bounds__(256) pv_rc_reference_kernel(const uint8_t* ref, uint64_t n, uint8_t* out) {
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
        out[i] = comp_up(ref[n - 1 - i]);
}

extern "C" int pv_rc_reference(const uint8_t* ref, uint64_t n, uint8_t* out, void* stream) {
    if (n == 0) return PV_OK;
    if (!ref || !out) { snprintf(g_cuda_err, sizeof g_cuda_err, "pv_rc_reference: arguments"); return PV_EARG; }
    pv_rc_reference_kernel<<<148 * 8, 256, 0, (cudaStream_t)stream>>>(ref, n, out);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) { snprintf(g_cuda_err, sizeof g_cuda_err, "%s", cudaGetErrorString(e)); return PV_ECUDA; }
    return PV_OK;
}

// ---------------------------------------------------------------- the checkpoint index: host side
extern "C" size_t pv_index_bytes(uint32_t Q, uint64_t nblocks, uint32_t ckpt_shift) {
    uint32_t qs = 0;
    while ((1u << qs) < Q) qs++;
    if ((1u << qs) != Q || ckpt_shift < 8 || ckpt_shift > qs || nblocks > (1ull << 40)) return 0;
    return (size_t)(nblocks << (qs - ckpt_shift)) * sizeof(pv_ckpt);
}

extern "C" int pv_index_build(const pv_dev_cohort* cohort, uint64_t nblocks, uint32_t ckpt_shift, pv_ckpt* out, uint64_t* nbad,
                              uint32_t* brun, uint16_t* cost, void* stream) {
    static_assert(sizeof(pv_ckpt) == 32, "pv_ckpt is two 16-byte words");
    const uint32_t Q = cohort ? cohort->Q : 0;
    if (!cohort || !(Q == 1024 || Q == 2048 || Q == 4096 || Q == 16384) || !pv_index_bytes(Q, nblocks, ckpt_shift) || !out ||
        ((uintptr_t)out & 15)) {
        snprintf(g_cuda_err, sizeof g_cuda_err, "pv_index_build: cohort, stride (256 to Q) or output (16-byte aligned)");
        return PV_EARG;
    }
    if ((cohort->packed && (!cohort->pref || !cohort->pruns || !cohort->pidx)) || (cohort->compact && (!cohort->groups || !cohort->btab)) ||
        (!cohort->packed && !cohort->ref) || (!cohort->compact && !cohort->blocks) || cohort->tab_max > PV_TAB_MAX_BYTES) {
        snprintf(g_cuda_err, sizeof g_cuda_err, "pv_index_build: the arrays of the cohort's resident form are missing");
        return PV_EARG;
    }
    if (cohort->ref_n >= (1ull << 38)) {                // diagonals are stored in 39 bits
        snprintf(g_cuda_err, sizeof g_cuda_err, "pv_index_build: reference longer than 2^38 bases");
        return PV_EARG;
    }
    if (nblocks == 0) return PV_OK;
    uint32_t qs = 0;
    while ((1u << qs) < Q) qs++;
    const unsigned grid = (unsigned)((nblocks + 127) / 128);
    const cudaStream_t st = (cudaStream_t)stream;
    unsigned long long* nb = (unsigned long long*)nbad;
    const int form = (cohort->packed ? 1 : 0) | (cohort->compact ? 2 : 0);
    switch (form) {
    case 0: pv_index_kernel<false, false><<<grid, 128, 0, st>>>(*cohort, nblocks, ckpt_shift, qs, (uint4*)out, nb, brun, cost); break;
    case 1: pv_index_kernel<true, false><<<grid, 128, 0, st>>>(*cohort, nblocks, ckpt_shift, qs, (uint4*)out, nb, brun, cost); break;
    case 2: pv_index_kernel<false, true><<<grid, 128, 0, st>>>(*cohort, nblocks, ckpt_shift, qs, (uint4*)out, nb, brun, cost); break;
    default: pv_index_kernel<true, true><<<grid, 128, 0, st>>>(*cohort, nblocks, ckpt_shift, qs, (uint4*)out, nb, brun, cost); break;
    }
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) { snprintf(g_cuda_err, sizeof g_cuda_err, "%s", cudaGetErrorString(e)); return PV_ECUDA; }
    return PV_OK;
}

// ---------------------------------------------------------------- the no-allocation variant (pv_windows_noalloc)
// Its scratch is this fixed array in device memory (PV_NOALLOC_SCRATCH_BYTES on every GPU that loads the library).
// Host code only sees a stand-in symbol for it: the device address is looked up once per device with
// cudaGetSymbolAddress and passed to the kernel like any other scratch pointer.
namespace {
static __device__ __align__(256) uint8_t g_noalloc_scratch[PV_NOALLOC_SCRATCH_BYTES];
std::atomic<void*> g_noalloc_addr[64];      // per device, filled by its first call (every thread would store the same)
}  // namespace

extern "C" int pv_windows_noalloc(const pv_dev_cohort* cohort, const int64_t* asm_index, const int64_t* start, int64_t n, int64_t W,
                                  const uint8_t* rc, int tokens, int apply_case, uint8_t* out, int32_t* status, void* stream) {
    const size_t need = pv_windows_work_bytes(cohort, n, W);
    if (need > (size_t)PV_NOALLOC_SCRATCH_BYTES) {
        snprintf(g_cuda_err, sizeof g_cuda_err, "pv_windows_noalloc: this call needs %zu bytes of scratch, more than the fixed %u; "
                 "split it into smaller calls (or use pv_windows with a caller buffer)", need, (unsigned)PV_NOALLOC_SCRATCH_BYTES);
        return PV_EARG;
    }
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= 64) {
        snprintf(g_cuda_err, sizeof g_cuda_err, "pv_windows_noalloc: current device: %s", e != cudaSuccess ? cudaGetErrorString(e) : "index >= 64");
        return PV_ECUDA;
    }
    void* addr = g_noalloc_addr[dev].load(std::memory_order_acquire);
    if (!addr) {                                             // set-up, once per device, with that device current
        e = cudaGetSymbolAddress(&addr, g_noalloc_scratch);
        if (e != cudaSuccess || !addr) {
            snprintf(g_cuda_err, sizeof g_cuda_err, "pv_windows_noalloc: scratch address: %s", cudaGetErrorString(e));
            return PV_ECUDA;
        }
        g_noalloc_addr[dev].store(addr, std::memory_order_release);
    }
    return pv_windows_ex(cohort, asm_index, start, n, W, rc, tokens, apply_case, 0u, out, status, nullptr, addr,
                         (size_t)PV_NOALLOC_SCRATCH_BYTES, stream);
}
