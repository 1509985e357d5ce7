// pv_fasta.cu - the whole-assembly checks on sm_100a: the FASTA file read over a decoded base stream in device memory
// (no copy of it is needed to hash it), the data-parallel half of its XXH3, per-block XXH3 checks and lower-case runs
// applied in place, with their host drivers. The reference rebuilds the FASTA and hashes it on the host
// (pv_core.cpp:138-176).
//
// Work per launch is HBM-bound byte work: each 1024-byte XXH3 block of the FASTA is one warp's (32 bytes a lane, so a
// lane pair holds one 64-byte stripe); the warp's partial sums meet by shuffles. The FASTA's bytes are produced on the
// fly from the record table (a binary search over the records, one division into lines): inside a record's full lines
// the warp reads the bases coalesced and regroups them through shared memory; at headers, record ends and short lines
// each lane steps byte by byte through header, bases and line ends.
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>

#include <atomic>
#include <thread>
#include <vector>

#include "panvram_b200.h"
#include "pv_xxh3.h"

namespace pvb { extern thread_local char g_cuda_err[256]; }

// from the xxHash library (libxxhash.so.0; its header is not installed): the secret of a seed (192 bytes), and the
// hash itself for inputs too short for the long-input path
extern "C" void XXH3_generateSecret_fromSeed(void* secret_buffer, uint64_t seed);
extern "C" uint64_t XXH3_64bits(const void* data, size_t len);

namespace {

using namespace pvx;

// ---------------------------------------------------------------- the FASTA as a byte stream over the records
struct FaPos {
    uint32_t r;                       // record
    uint64_t fo, x, len, hdr_off;     // its start, the stream index of the next base, its length, its header's bytes
    uint32_t hlen, lw;
    uint64_t hpos;                    // in the header line: byte index ('>' is 0, the '\n' hlen + 1)
    uint64_t done, ll, col;           // in the bases: bases before this line, this line's length, column
    bool hdr;
};
__device__ __forceinline__ void fa_load(const pv_fasta_view& V, FaPos& f, uint32_t r) {
    const pv_fasta_rec* R = V.recs + r;
    f.r = r;
    f.fo = __ldg(&R->fasta_off);
    f.x = __ldg(&R->boff);
    f.len = __ldg(&R->len);
    f.hdr_off = __ldg(&R->hdr_off);
    f.hlen = __ldg(&R->hdr_len);
    f.lw = __ldg(&R->line_width);
    f.hdr = true; f.hpos = 0;
}
__device__ __forceinline__ void fa_line(FaPos& f) { f.ll = f.len - f.done < f.lw ? f.len - f.done : f.lw; f.col = 0; }
// position f at FASTA byte p (< fasta_len)
__device__ void fa_seek(const pv_fasta_view& V, FaPos& f, uint64_t p) {
    uint32_t lo = 0, hi = (uint32_t)V.nrec;             // records[lo].fasta_off <= p (records[0] starts at 0)
    while (hi - lo > 1) {
        const uint32_t mid = (lo + hi) >> 1;
        if (__ldg(&V.recs[mid].fasta_off) <= p) lo = mid; else hi = mid;
    }
    fa_load(V, f, lo);
    const uint64_t local = p - f.fo, h = (uint64_t)f.hlen + 2;
    if (local < h) { f.hpos = local; return; }
    const uint64_t q = local - h, line = q / ((uint64_t)f.lw + 1), col = q - line * ((uint64_t)f.lw + 1);
    f.hdr = false;
    f.done = line * f.lw;
    fa_line(f);
    f.col = col;
    f.x += f.done + (col < f.ll ? col : f.ll);
}
// the byte at f, then f moves to the next one
__device__ __forceinline__ uint32_t fa_next(const pv_fasta_view& V, FaPos& f) {
    uint32_t b;
    if (f.hdr) {
        const uint64_t h = (uint64_t)f.hlen + 2;
        b = f.hpos == 0 ? (uint32_t)'>' : f.hpos == h - 1 ? (uint32_t)'\n' : (uint32_t)__ldg(V.hdrs + f.hdr_off + f.hpos - 1);
        if (++f.hpos == h) {
            if (f.len) { f.hdr = false; f.done = 0; fa_line(f); }
            else if (f.r + 1 < V.nrec) fa_load(V, f, f.r + 1);
        }
    } else if (f.col < f.ll) {
        b = __ldg(V.bases + f.x);
        f.x++; f.col++;
    } else {
        b = '\n';
        f.done += f.ll;
        if (f.done < f.len) fa_line(f);
        else if (f.r + 1 < V.nrec) fa_load(V, f, f.r + 1);
    }
    return b;
}
// FASTA bytes [p, p + 32) as 4 little-endian words (p + 32 <= fasta_len)
__device__ __forceinline__ void fa_read32(const pv_fasta_view& V, uint64_t p, uint64_t w[4]) {
    FaPos f;
    fa_seek(V, f, p);
#pragma unroll
    for (int j = 0; j < 4; j++) {
        uint64_t v = 0;
#pragma unroll
        for (int k = 0; k < 8; k++) v |= (uint64_t)fa_next(V, f) << (8 * k);
        w[j] = v;
    }
}

// ---------------------------------------------------------------- XXH3 block sums over a warp
// lane l holds 32 bytes of a 1024-byte block: words 4 (l & 1) .. 4 (l & 1) + 3 of stripe l >> 1. Its share of the
// accumulate steps lands on accumulators 4 (l & 1) .. + 3 (acc[i] and acc[i ^ 1] stay in the same half); after the
// xor-shuffles over lanes of the same parity every lane holds its half's four sums.
__device__ __forceinline__ void block_sums(const uint64_t w[4], const uint64_t key[4], bool on, uint64_t p[4]) {
#pragma unroll
    for (int j = 0; j < 4; j++) p[j] = on ? mul32x32(w[j] ^ key[j]) + w[j ^ 1] : 0;
#pragma unroll
    for (int o = 2; o < 32; o <<= 1)
#pragma unroll
        for (int j = 0; j < 4; j++) p[j] += __shfl_xor_sync(0xFFFFFFFFu, p[j], o);
}
__device__ __forceinline__ void lane_keys(const uint64_t* kw, int lane, uint64_t key[4]) {
#pragma unroll
    for (int j = 0; j < 4; j++) key[j] = kw[(lane >> 1) + 4 * (lane & 1) + j];    // secret word s + i
}

// One warp, the 1024 FASTA bytes [B, B + 1024) (B + 1024 <= fasta_len): lane l gets bytes [B + 32 l, B + 32 l + 32)
// as 4 little-endian words. When the block lies inside full lines of one record's bases (the common case: records are
// long, lines at least 32 wide) the warp steps through it coalesced - byte B + 32 j + l by lane l at step j, a line
// end crossed at most once per step - and regroups the bytes through shared memory; otherwise each lane seeks and
// steps on its own.
__device__ __forceinline__ void fa_block1k(const pv_fasta_view& V, uint64_t B, uint8_t* stage, int lane, uint64_t w[4]) {
    uint32_t lo = 0, hi = (uint32_t)V.nrec;              // the record holding B (warp-uniform)
    while (hi - lo > 1) {
        const uint32_t mid = (lo + hi) >> 1;
        if (__ldg(&V.recs[mid].fasta_off) <= B) lo = mid; else hi = mid;
    }
    const pv_fasta_rec* R = V.recs + lo;
    const uint64_t len = __ldg(&R->len), lw = __ldg(&R->line_width);
    const uint64_t seq = __ldg(&R->fasta_off) + __ldg(&R->hdr_len) + 2;
    const uint64_t last = lw && len ? seq + ((len + lw - 1) / lw - 1) * (lw + 1) : 0;   // where the last (maybe short) line starts
    if (lw >= 32 && B >= seq && B + BLOCK <= last) {
        const uint64_t q = B + lane - seq, line = q / (lw + 1);
        uint32_t col = (uint32_t)(q - line * (lw + 1));
        const uint32_t L = (uint32_t)lw;
        const uint8_t* x = V.bases + __ldg(&R->boff) + line * lw + col;
#pragma unroll 8
        for (int j = 0; j < 32; j++) {
            stage[32 * j + lane] = col == L ? (uint8_t)'\n' : __ldg(x);
            const bool wrap = col + 32 > L;
            col = wrap ? col + 32 - (L + 1) : col + 32;
            x += wrap ? 31 : 32;
        }
        __syncwarp();
        const ulonglong2 a = *(const ulonglong2*)(stage + 32 * lane), c = *(const ulonglong2*)(stage + 32 * lane + 16);
        w[0] = a.x; w[1] = a.y; w[2] = c.x; w[3] = c.y;
        __syncwarp();
    } else {
        fa_read32(V, B + 32 * lane, w);
    }
}

constexpr int FA_WARPS = 8;      // warps per CTA of the FASTA kernels (256 threads), each with a 1 KB staging row

__global__ void __launch_bounds__(256) pv_fasta_xxh3_kernel(const __grid_constant__ pv_fasta_view V, uint64_t blk0,
                                                            uint64_t nblk, uint64_t* contrib) {
    __shared__ __align__(16) uint8_t stage[FA_WARPS][BLOCK];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    uint64_t key[4];
    lane_keys(V.keys, lane, key);
    const uint64_t nw = (uint64_t)gridDim.x * FA_WARPS;
    for (uint64_t k = (uint64_t)blockIdx.x * FA_WARPS + warp; k < nblk; k += nw) {
        uint64_t w[4], p[4];
        fa_block1k(V, (blk0 + k) * BLOCK, stage[warp], lane, w);
        block_sums(w, key, true, p);
        if (lane < 4) {                          // lane-major: accumulator j's sums are contrib[j * nblk ...]
            const int j0 = 4 * (lane & 1) + 2 * (lane >> 1);
            contrib[(uint64_t)j0 * nblk + k] = p[2 * (lane >> 1)];
            contrib[(uint64_t)(j0 + 1) * nblk + k] = p[2 * (lane >> 1) + 1];
        }
    }
}

// FASTA bytes [p0, p1) into out: one warp per 1024 bytes (the last, partial kilobyte byte by byte)
__global__ void __launch_bounds__(256) pv_fasta_bytes_kernel(const __grid_constant__ pv_fasta_view V, uint64_t p0, uint64_t p1,
                                                             uint8_t* out) {
    __shared__ __align__(16) uint8_t stage[FA_WARPS][BLOCK];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint64_t nw = (uint64_t)gridDim.x * FA_WARPS, nk = (p1 - p0 + BLOCK - 1) / BLOCK;
    for (uint64_t k = (uint64_t)blockIdx.x * FA_WARPS + warp; k < nk; k += nw) {
        const uint64_t B = p0 + k * BLOCK;
        if (B + BLOCK <= p1) {
            uint64_t w[4];
            fa_block1k(V, B, stage[warp], lane, w);
            ulonglong2* o = (ulonglong2*)(out + k * BLOCK + 32 * lane);
            o[0] = make_ulonglong2(w[0], w[1]);
            o[1] = make_ulonglong2(w[2], w[3]);
        } else {
            const uint64_t q0 = B + 32 * lane;
            if (q0 < p1) {
                FaPos f;
                fa_seek(V, f, q0);
                const uint64_t q1 = q0 + 32 < p1 ? q0 + 32 : p1;
                for (uint64_t q = q0; q < q1; q++) out[q - p0] = (uint8_t)fa_next(V, f);
            }
        }
    }
}

// ---------------------------------------------------------------- per-block XXH3 (one warp per block)
struct BlockHashParams {
    const uint8_t* bases; uint64_t nbases, nb; uint32_t Q;
    const uint64_t* want; int64_t* first_bad;
    uint64_t keys[40];
};
__device__ __forceinline__ uint64_t lane_total(const uint64_t p[4], int acc_lane) {
    // the sum for accumulator acc_lane (0..7) from a lane of parity acc_lane >> 2
    const int src = acc_lane >> 2, j = acc_lane & 3;
    const uint64_t t0 = __shfl_sync(0xFFFFFFFFu, p[0], src), t1 = __shfl_sync(0xFFFFFFFFu, p[1], src);
    const uint64_t t2 = __shfl_sync(0xFFFFFFFFu, p[2], src), t3 = __shfl_sync(0xFFFFFFFFu, p[3], src);
    return j == 0 ? t0 : j == 1 ? t1 : j == 2 ? t2 : t3;
}
__global__ void __launch_bounds__(256) pv_block_xxh3_kernel(const __grid_constant__ BlockHashParams P) {
    const int lane = threadIdx.x & 31, ai = lane & 7;    // lanes 0..7 keep accumulator ai (the others mirror them)
    uint64_t key[4];
    lane_keys(P.keys, lane, key);
    const uint64_t nw = (uint64_t)gridDim.x * (blockDim.x >> 5);
    for (uint64_t b = (uint64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); b < P.nb; b += nw) {
        const uint64_t L = P.nbases - b * P.Q < P.Q ? P.nbases - b * P.Q : P.Q;
        if (L < LONG_INPUT) continue;                                   // (warp-uniform)
        const uint8_t* in = P.bases + b * P.Q;
        uint64_t acc = acc_init(ai), p[4], w[4];
        const uint64_t nfull = (L - 1) / BLOCK;
        for (uint64_t k = 0; k <= nfull; k++) {
            // full blocks, then the stripes of the partial block wholly before byte L - 1
            const bool on = k < nfull || (uint64_t)(lane >> 1) < ((L - 1) - BLOCK * nfull) / STRIPE;
            if (on) {
                const ulonglong2* s = (const ulonglong2*)(in + k * BLOCK + 32 * lane);   // Q is a multiple of 1024
                const ulonglong2 a = __ldg(s), c = __ldg(s + 1);
                w[0] = a.x; w[1] = a.y; w[2] = c.x; w[3] = c.y;
            }
            block_sums(w, key, on, p);
            acc += lane_total(p, ai);
            if (k < nfull) acc = scramble(acc, P.keys[16 + ai]);
        }
        // the last 64 bytes: word ai by lane ai (byte loads: L - 64 has any alignment)
        uint64_t d = 0;
#pragma unroll
        for (int k = 0; k < 8; k++) d |= (uint64_t)__ldg(in + L - STRIPE + 8 * ai + k) << (8 * k);
        acc += mul32x32(d ^ P.keys[24 + ai]) + __shfl_xor_sync(0xFFFFFFFFu, d, 1);
        // merge: pairs (2j, 2j + 1) folded on even lanes, summed into lane 0
        const uint64_t m = acc ^ P.keys[32 + ai];
        const uint64_t mo = __shfl_down_sync(0xFFFFFFFFu, m, 1);
        uint64_t f = (lane < 8 && (lane & 1) == 0) ? fold64(m, mo) : 0;
        f += __shfl_down_sync(0xFFFFFFFFu, f, 2);
        f += __shfl_down_sync(0xFFFFFFFFu, f, 4);
        if (lane == 0) {
            const uint64_t h = avalanche(L * PRIME64_1 + f);
            if (h != __ldg(P.want + b)) atomicMin((unsigned long long*)P.first_bad, (unsigned long long)b);
        }
    }
}

// ---------------------------------------------------------------- lower-case runs (one warp per run)
__global__ void __launch_bounds__(256) pv_apply_case_kernel(const pv_asm_rec* asms, const uint64_t* low, int64_t a, uint8_t* bases,
                                                            uint64_t nbases) {
    const int lane = threadIdx.x & 31;
    const uint64_t base = __ldg(&asms[a].low_base), cnt = __ldg(&asms[a].low_cnt);
    const uint64_t nw = (uint64_t)gridDim.x * (blockDim.x >> 5);
    for (uint64_t r = (uint64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < cnt; r += nw) {
        const uint64_t s = __ldg(low + 2 * (base + r)), e0 = __ldg(low + 2 * (base + r) + 1), e = e0 < nbases ? e0 : nbases;
        for (uint64_t x = s + lane; x < e; x += 32) bases[x] |= 0x20;
    }
}

int fail(int code, const char* what) {
    snprintf(pvb::g_cuda_err, sizeof pvb::g_cuda_err, "%s", what);
    return code;
}
int launched(const char* what) {
    const cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) return PV_OK;
    snprintf(pvb::g_cuda_err, sizeof pvb::g_cuda_err, "%s: %s", what, cudaGetErrorString(e));
    return PV_ECUDA;
}
unsigned grid_for(uint64_t warps) {
    const uint64_t ctas = (warps + 7) / 8;
    return (unsigned)(ctas < 148 * 16 ? (ctas ? ctas : 1) : 148 * 16);
}

// ---------------------------------------------------------------- host side: the secret, the serial chain, the finish
// XXH3's default secret, from the xxHash library (seed 0 gives the default secret itself), as the device reads it
const Keys& xxh3_keys() {
    static Keys k;
    static bool ready = [] {
        uint8_t secret[SECRET_BYTES];
        XXH3_generateSecret_fromSeed(secret, 0);
        keys_from_secret(secret, &k);
        return true;
    }();
    (void)ready;
    return k;
}
void keys40(const Keys& k, uint64_t out[40]) {
    memcpy(out, k.w, 24 * 8); memcpy(out + 24, k.last, 8 * 8); memcpy(out + 32, k.merge, 8 * 8);
}
// the serial chain over n block sums: acc = scramble(acc + sum) per block (sums block-major, 8 per block)
void scan_blocks(uint64_t acc[8], const uint64_t* sums, uint64_t n, const Keys& k) {
    uint64_t a[8];
    for (int i = 0; i < 8; i++) a[i] = acc[i];
    for (uint64_t b = 0; b < n; b++)
        for (int i = 0; i < 8; i++) a[i] = scramble(a[i] + sums[8 * b + i], k.w[16 + i]);
    for (int i = 0; i < 8; i++) acc[i] = a[i];
}
// the same for accumulators j0 .. j0 + 3 over lane-major sums (accumulator j's n sums at sums + j * n)
void scan_lanes4(uint64_t acc[8], const uint64_t* sums, uint64_t n, int j0, const Keys& k) {
    uint64_t a0 = acc[j0], a1 = acc[j0 + 1], a2 = acc[j0 + 2], a3 = acc[j0 + 3];
    const uint64_t k0 = k.w[16 + j0], k1 = k.w[17 + j0], k2 = k.w[18 + j0], k3 = k.w[19 + j0];
    const uint64_t *s0 = sums + (uint64_t)j0 * n, *s1 = s0 + n, *s2 = s1 + n, *s3 = s2 + n;
    for (uint64_t b = 0; b < n; b++) {
        a0 = scramble(a0 + s0[b], k0); a1 = scramble(a1 + s1[b], k1);
        a2 = scramble(a2 + s2[b], k2); a3 = scramble(a3 + s3[b], k3);
    }
    acc[j0] = a0; acc[j0 + 1] = a1; acc[j0 + 2] = a2; acc[j0 + 3] = a3;
}
// after the full blocks: the partial block's stripes, the last stripe, the merge. tail = input bytes [t0, len).
uint64_t finish(uint64_t acc[8], const uint8_t* tail, uint64_t t0, uint64_t len, const Keys& k) {
    const uint64_t nfull = (len - 1) / BLOCK, ns = ((len - 1) - BLOCK * nfull) / STRIPE;
    for (uint64_t s = 0; s < ns; s++) stripe(acc, tail + (BLOCK * nfull + STRIPE * s - t0), k.w + s);
    stripe(acc, tail + (len - STRIPE - t0), k.last);
    return merge(acc, k.merge, len);
}
uint64_t tail_start(uint64_t len) {
    const uint64_t a = BLOCK * ((len - 1) / BLOCK), b = len - STRIPE;
    return a < b ? a : b;
}

int from_core(int code) {
    if (code != PV_OK) snprintf(pvb::g_cuda_err, sizeof pvb::g_cuda_err, "%s", pv_last_error());
    return code;
}
int cuda_ok(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return PV_OK;
    snprintf(pvb::g_cuda_err, sizeof pvb::g_cuda_err, "%s: %s", what, cudaGetErrorString(e));
    return PV_ECUDA;
}
#define PV_TRY(x) do { const int rc_ = (x); if (rc_ != PV_OK) return rc_; } while (0)

// scratch layout of the host drivers: record table | header bytes | two block-sum chunks | tail | block hashes | word
constexpr uint64_t CHUNK = 1ull << 16;          // XXH3 blocks per chunk by default (64 MiB of FASTA, 4 MiB of sums)
constexpr uint64_t TAIL_CAP = 2048;
uint64_t up256(uint64_t x) { return (x + 255) & ~255ull; }
struct Scratch { pv_fasta_rec* recs; uint8_t* hdrs; uint64_t* sums[2]; uint8_t* tail; uint64_t* want; int64_t* word; uint64_t bytes; };
Scratch scratch_of(uint8_t* w, uint64_t nrec, uint64_t hdr_bytes, uint64_t nhash, uint64_t chunk = CHUNK) {
    Scratch s;
    uint64_t o = 0;
    s.recs = (pv_fasta_rec*)(w + o); o += up256(nrec * sizeof(pv_fasta_rec));
    s.hdrs = w + o; o += up256(hdr_bytes + 1);
    s.sums[0] = (uint64_t*)(w + o); o += chunk * 64;
    s.sums[1] = (uint64_t*)(w + o); o += chunk * 64;
    s.tail = w + o; o += TAIL_CAP;
    s.want = (uint64_t*)(w + o); o += up256(nhash * 8);
    s.word = (int64_t*)(w + o); o += 256;
    s.bytes = o;
    return s;
}

// the view of assembly i's FASTA over `bases`, its record table uploaded into the scratch
int make_view(const pv_core* c, int64_t i, const uint8_t* bases, uint64_t nbases, void* work, size_t work_bytes, cudaStream_t st,
              pv_fasta_view* v, Scratch* s, uint64_t chunk = CHUNK) {
    pv_asm_info info;
    PV_TRY(from_core(pv_core_info(c, i, &info)));
    if (nbases != info.bases) return fail(PV_EARG, "bases: the assembly's decoded stream (device)");
    if (!bases || ((uintptr_t)bases & 15) || !work || ((uintptr_t)work & 15)) return fail(PV_EARG, "device buffers: 16-byte aligned");
    uint64_t nrec, hb, flen;
    PV_TRY(from_core(pv_core_fasta_layout(c, i, nullptr, 0, nullptr, 0, &nrec, &hb, &flen)));
    const uint64_t* hashes; uint64_t nh; uint32_t Q;
    PV_TRY(from_core(pv_core_block_hashes(c, i, &hashes, &nh, &Q)));
    *s = scratch_of((uint8_t*)work, nrec, hb, nh, chunk);
    if (work_bytes < s->bytes) return fail(PV_EARG, "work buffer smaller than pv_core_device_check_work_bytes()");
    if (nrec == 0) return fail(PV_EARG, "assembly without contigs");
    std::vector<pv_fasta_rec> recs(nrec);
    std::vector<uint8_t> hdrs(hb + 1);
    PV_TRY(from_core(pv_core_fasta_layout(c, i, recs.data(), nrec, hdrs.data(), hb + 1, &nrec, &hb, &flen)));
    for (uint64_t r = 0; r < nrec; r++)          // every read the kernels make stays inside the stream and the headers
        if (recs[r].boff > nbases || recs[r].len > nbases - recs[r].boff || (r && recs[r].fasta_off <= recs[r - 1].fasta_off))
            return fail(PV_EFORMAT, "contig table outside the assembly's stream");
    PV_TRY(cuda_ok(cudaMemcpyAsync(s->recs, recs.data(), nrec * sizeof(pv_fasta_rec), cudaMemcpyHostToDevice, st), "record table"));
    PV_TRY(cuda_ok(cudaMemcpyAsync(s->hdrs, hdrs.data(), hb + 1, cudaMemcpyHostToDevice, st), "headers"));
    PV_TRY(cuda_ok(cudaStreamSynchronize(st), "record table"));     // (the host vectors go out of scope)
    v->recs = s->recs; v->hdrs = s->hdrs; v->bases = bases;
    v->nrec = nrec; v->nbases = nbases; v->fasta_len = flen;
    keys40(xxh3_keys(), v->keys);
    return PV_OK;
}

struct PinnedPair {
    uint64_t* p = nullptr;
    cudaEvent_t ev[2] = {nullptr, nullptr};
    ~PinnedPair() {
        if (p) cudaFreeHost(p);
        for (auto e : ev) if (e) cudaEventDestroy(e);
    }
};

}  // namespace

extern "C" {

int pv_fasta_xxh3_blocks(const pv_fasta_view* v, uint64_t blk0, uint64_t nblk, uint64_t* contrib, void* stream) {
    if (!v || !contrib || ((uintptr_t)contrib & 15)) return fail(PV_EARG, "pv_fasta_xxh3_blocks: arguments");
    if (nblk == 0) return PV_OK;
    if (v->nrec == 0 || v->nrec >= (1ull << 32) || (blk0 + nblk) * BLOCK > v->fasta_len)
        return fail(PV_EARG, "pv_fasta_xxh3_blocks: blocks outside the FASTA");
    pv_fasta_xxh3_kernel<<<grid_for(nblk), 256, 0, (cudaStream_t)stream>>>(*v, blk0, nblk, contrib);
    return launched("pv_fasta_xxh3_kernel");
}

int pv_fasta_bytes(const pv_fasta_view* v, uint64_t p0, uint64_t p1, uint8_t* out, void* stream) {
    if (!v || !out || ((uintptr_t)out & 15) || p0 > p1 || p1 > v->fasta_len) return fail(PV_EARG, "pv_fasta_bytes: arguments");
    if (p0 == p1) return PV_OK;
    if (v->nrec == 0 || v->nrec >= (1ull << 32)) return fail(PV_EARG, "pv_fasta_bytes: records");
    pv_fasta_bytes_kernel<<<grid_for((p1 - p0 + BLOCK - 1) / BLOCK), 256, 0, (cudaStream_t)stream>>>(*v, p0, p1, out);
    return launched("pv_fasta_bytes_kernel");
}

int pv_block_xxh3_check(const uint8_t* bases, uint64_t nbases, uint32_t Q, const uint64_t* want, const uint64_t* keys40,
                        int64_t* first_bad, void* stream) {
    if (!(Q == 1024 || Q == 2048 || Q == 4096 || Q == 16384) || !keys40 || !first_bad) return fail(PV_EARG, "pv_block_xxh3_check: arguments");
    if (nbases == 0) return PV_OK;
    if (!bases || !want || ((uintptr_t)bases & 15)) return fail(PV_EARG, "pv_block_xxh3_check: arguments");
    BlockHashParams P;
    P.bases = bases; P.nbases = nbases; P.nb = (nbases + Q - 1) / Q; P.Q = Q; P.want = want; P.first_bad = first_bad;
    memcpy(P.keys, keys40, sizeof P.keys);
    pv_block_xxh3_kernel<<<grid_for(P.nb), 256, 0, (cudaStream_t)stream>>>(P);
    return launched("pv_block_xxh3_kernel");
}

int pv_apply_case_device(const pv_dev_cohort* cohort, int64_t asm_index, uint64_t max_runs, uint8_t* bases, uint64_t nbases,
                         void* stream) {
    if (!cohort || asm_index < 0 || asm_index >= cohort->nasm) return fail(PV_EARG, "pv_apply_case_device: arguments");
    if (max_runs == 0 || nbases == 0) return PV_OK;
    if (!bases || !cohort->low || !cohort->asms) return fail(PV_EARG, "pv_apply_case_device: arguments");
    pv_apply_case_kernel<<<grid_for(max_runs), 256, 0, (cudaStream_t)stream>>>(cohort->asms, cohort->low, asm_index, bases, nbases);
    return launched("pv_apply_case_kernel");
}

size_t pv_core_device_check_work_bytes(const pv_core* c, int64_t i) {
    uint64_t nrec, hb, flen, nh; const uint64_t* h; uint32_t Q;
    if (pv_core_fasta_layout(c, i, nullptr, 0, nullptr, 0, &nrec, &hb, &flen) != PV_OK) return 0;
    if (pv_core_block_hashes(c, i, &h, &nh, &Q) != PV_OK) return 0;
    return scratch_of(nullptr, nrec, hb, nh).bytes;
}

int pv_core_fasta_xxh3_device(const pv_core* c, int64_t i, const uint8_t* bases, uint64_t nbases, uint64_t chunk_blocks, void* work,
                              size_t work_bytes, void* stream, uint64_t* out_hash) {
    const cudaStream_t st = (cudaStream_t)stream;
    const uint64_t CH = chunk_blocks ? (chunk_blocks < CHUNK ? chunk_blocks : CHUNK) : CHUNK;
    pv_fasta_view v; Scratch s;
    PV_TRY(make_view(c, i, bases, nbases, work, work_bytes, st, &v, &s, CH));
    const uint64_t len = v.fasta_len;
    const Keys& k = xxh3_keys();
    if (len < LONG_INPUT) {                         // short inputs take other XXH3 paths: the bytes to the library
        uint8_t b[LONG_INPUT];
        PV_TRY(pv_fasta_bytes(&v, 0, len, s.tail, stream));
        PV_TRY(cuda_ok(cudaMemcpyAsync(b, s.tail, len, cudaMemcpyDeviceToHost, st), "FASTA bytes"));
        PV_TRY(cuda_ok(cudaStreamSynchronize(st), "FASTA bytes"));
        *out_hash = XXH3_64bits(b, len);
        return PV_OK;
    }
    // block sums on the device a chunk at a time, copied back into two pinned buffers; while the device works on chunk
    // j, the host runs the scramble chain over chunk j - 1: accumulators 0-3 on this thread, 4-7 on a helper (the chain
    // is bound by reading the sums and by each step's latency, so two threads take about half the time)
    const uint64_t nfull = (len - 1) / BLOCK, nch = (nfull + CH - 1) / CH;
    uint64_t acc[8];
    for (int j = 0; j < 8; j++) acc[j] = acc_init(j);
    PinnedPair pp;
    if (nch) {
        PV_TRY(cuda_ok(cudaMallocHost(&pp.p, 2 * CH * 64), "pinned block sums"));
        for (auto& e : pp.ev) PV_TRY(cuda_ok(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "event"));
    }
    auto blocks_in = [&](uint64_t j) { const uint64_t b0 = j * CH; return nfull - b0 < CH ? nfull - b0 : CH; };
    std::atomic<int64_t> issued{-1};               // the last chunk whose sums are on their way to the host
    std::atomic<int64_t> helper_done{-1};          // the last chunk the helper has scanned
    std::atomic<bool> stop{false};
    std::atomic<int> helper_err{0};
    std::thread helper([&] {
        for (uint64_t j = 0; j < nch; j++) {
            while ((int64_t)issued.load() < (int64_t)j && !stop.load()) std::this_thread::yield();
            if (stop.load()) return;
            if (cudaEventSynchronize(pp.ev[j & 1]) != cudaSuccess) { helper_err = 1; return; }
            scan_lanes4(acc, pp.p + (j & 1) * CH * 8, blocks_in(j), 4, k);
            helper_done = (int64_t)j;
        }
    });
    int rc = PV_OK;
    for (uint64_t j = 0; j <= nch && rc == PV_OK; j++) {
        if (j < nch) {
            // buffer j & 1 held chunk j - 2: both threads must be done with it
            while (j >= 2 && helper_done.load() < (int64_t)j - 2 && !helper_err.load()) std::this_thread::yield();
            if (helper_err.load()) { rc = fail(PV_ECUDA, "block sums: event"); break; }
            const uint64_t nb = blocks_in(j);
            rc = pv_fasta_xxh3_blocks(&v, j * CH, nb, s.sums[j & 1], stream);
            if (rc == PV_OK)
                rc = cuda_ok(cudaMemcpyAsync(pp.p + (j & 1) * CH * 8, s.sums[j & 1], nb * 64, cudaMemcpyDeviceToHost, st), "block sums");
            if (rc == PV_OK) rc = cuda_ok(cudaEventRecord(pp.ev[j & 1], st), "event");
            if (rc == PV_OK) issued = (int64_t)j;
        }
        if (j > 0 && rc == PV_OK) {
            rc = cuda_ok(cudaEventSynchronize(pp.ev[(j - 1) & 1]), "block sums");
            if (rc == PV_OK) scan_lanes4(acc, pp.p + ((j - 1) & 1) * CH * 8, blocks_in(j - 1), 0, k);
        }
    }
    if (rc != PV_OK) stop = true;
    helper.join();
    if (rc != PV_OK) return rc;
    if (helper_err.load()) return fail(PV_ECUDA, "block sums: event");
    const uint64_t t0 = tail_start(len);
    uint8_t tail[TAIL_CAP];
    PV_TRY(pv_fasta_bytes(&v, t0, len, s.tail, stream));
    PV_TRY(cuda_ok(cudaMemcpyAsync(tail, s.tail, len - t0, cudaMemcpyDeviceToHost, st), "FASTA tail"));
    PV_TRY(cuda_ok(cudaStreamSynchronize(st), "FASTA tail"));
    *out_hash = finish(acc, tail, t0, len, k);
    return PV_OK;
}

int pv_core_fasta_write_device(const pv_core* c, int64_t i, const uint8_t* bases, uint64_t nbases, uint8_t* out, uint64_t cap,
                               void* work, size_t work_bytes, void* stream, uint64_t* size) {
    uint64_t nrec, hb, flen;
    PV_TRY(from_core(pv_core_fasta_layout(c, i, nullptr, 0, nullptr, 0, &nrec, &hb, &flen)));
    *size = flen;
    if (!out) return PV_OK;
    if (cap < flen || ((uintptr_t)out & 15)) return fail(PV_EARG, "FASTA buffer: too small or not 16-byte aligned");
    const cudaStream_t st = (cudaStream_t)stream;
    pv_fasta_view v; Scratch s;
    PV_TRY(make_view(c, i, bases, nbases, work, work_bytes, st, &v, &s));
    PV_TRY(pv_fasta_bytes(&v, 0, flen, out, stream));
    return cuda_ok(cudaStreamSynchronize(st), "FASTA bytes");
}

int pv_core_check_block_hashes_device(const pv_core* c, int64_t i, const uint8_t* upper, uint64_t nbases, void* work, size_t work_bytes,
                                      void* stream, int64_t* first_bad) {
    *first_bad = -1;
    const cudaStream_t st = (cudaStream_t)stream;
    pv_fasta_view v; Scratch s;
    PV_TRY(make_view(c, i, upper, nbases, work, work_bytes, st, &v, &s));
    const uint64_t* hashes; uint64_t nh; uint32_t Q;
    PV_TRY(from_core(pv_core_block_hashes(c, i, &hashes, &nh, &Q)));
    if (nh == 0 || nbases == 0) return PV_OK;
    if (nh != (nbases + Q - 1) / Q) return fail(PV_EFORMAT, "block hash count");
    int64_t w = INT64_MAX;
    PV_TRY(cuda_ok(cudaMemcpyAsync(s.want, hashes, nh * 8, cudaMemcpyHostToDevice, st), "block hashes"));
    PV_TRY(cuda_ok(cudaMemcpyAsync(s.word, &w, 8, cudaMemcpyHostToDevice, st), "block hashes"));
    PV_TRY(pv_block_xxh3_check(upper, nbases, Q, s.want, v.keys, s.word, stream));
    PV_TRY(cuda_ok(cudaMemcpyAsync(&w, s.word, 8, cudaMemcpyDeviceToHost, st), "block hashes"));
    // the last block, if it is too short for the long-input path: its bytes to the library
    const uint64_t lb = nh - 1, L = nbases - lb * Q;
    uint8_t b[LONG_INPUT];
    if (L < LONG_INPUT) PV_TRY(cuda_ok(cudaMemcpyAsync(b, upper + lb * Q, L, cudaMemcpyDeviceToHost, st), "last block"));
    PV_TRY(cuda_ok(cudaStreamSynchronize(st), "block hashes"));
    if (L < LONG_INPUT && XXH3_64bits(b, L) != hashes[lb] && (int64_t)lb < w) w = (int64_t)lb;
    *first_bad = w == INT64_MAX ? -1 : w;
    return PV_OK;
}

int pv_xxh3_64_long_host(const void* data, uint64_t len, uint64_t* out_hash) {
    if (!data || len < LONG_INPUT) return fail(PV_EARG, "pv_xxh3_64_long_host: more than 240 bytes");
    const uint8_t* in = (const uint8_t*)data;
    const Keys& k = xxh3_keys();
    uint64_t acc[8];
    for (int j = 0; j < 8; j++) acc[j] = acc_init(j);
    const uint64_t nfull = (len - 1) / BLOCK;
    std::vector<uint64_t> sums(8);
    for (uint64_t b = 0; b < nfull; b++) {          // each block's sum from zero accumulators, as the device forms it
        for (auto& x : sums) x = 0;
        for (int s = 0; s < STRIPES_PER_BLOCK; s++) stripe(sums.data(), in + b * BLOCK + s * STRIPE, k.w + s);
        scan_blocks(acc, sums.data(), 1, k);
    }
    const uint64_t t0 = tail_start(len);
    *out_hash = finish(acc, in + t0, t0, len, k);
    return PV_OK;
}

}  // extern "C"
