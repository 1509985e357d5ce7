// pv_synth.cpp - synthetic pangenome cohorts written as refrel3 v1 archives (test and benchmark data, not part of the
// decode path). A reference is generated (uniform ACGT, N runs, soft-masked runs in its FASTA); each assembly is that
// reference with SNVs, indels and structural variants applied, fragmented into contigs (some reverse-complemented),
// with its own soft-masked runs. Because the generator knows every edit, it emits the refrel3 events directly - a
// copy per reference segment of 12 bases or more, literals for everything else - instead of searching for matches
// as the reference encoder (tools/rr3bench/refrel3v1.cpp) does; the archive obeys the same format (FORMAT.md 1-4):
// same grammar and contexts as refrel3.h's decoder, static per-assembly tables normalised to 4096, byte-wise rANS
// with the state in [2^16, 2^24) encoded backwards from 2^16, zstd meta, XXH3 header / block / FASTA hashes.
#include <openssl/sha.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <random>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

#include "../csrc/pv_layout.h"

extern "C" {
size_t ZSTD_compressBound(size_t srcSize);
size_t ZSTD_compress(void* dst, size_t dstCapacity, const void* src, size_t srcSize, int compressionLevel);
unsigned ZSTD_isError(size_t code);
uint64_t XXH3_64bits(const void* data, size_t len);
typedef struct XXH3_state_s XXH3_state_t;
XXH3_state_t* XXH3_createState(void);
int XXH3_freeState(XXH3_state_t* s);
int XXH3_64bits_reset(XXH3_state_t* s);
int XXH3_64bits_update(XXH3_state_t* s, const void* p, size_t n);
uint64_t XXH3_64bits_digest(const XXH3_state_t* s);
}

namespace {
using namespace pvb;

thread_local std::string g_err;

// ---------------------------------------------------------------- random numbers (splitmix64 seeding, xoshiro256**)
struct Rng {
    uint64_t s[4];
    explicit Rng(uint64_t seed) {
        for (int i = 0; i < 4; i++) { seed += 0x9E3779B97F4A7C15ull; uint64_t z = seed; z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
            z = (z ^ (z >> 27)) * 0x94D049BB133111EBull; s[i] = z ^ (z >> 31); }
    }
    static uint64_t rotl(uint64_t x, int k) { return (x << k) | (x >> (64 - k)); }
    uint64_t next() {
        const uint64_t r = rotl(s[1] * 5, 7) * 9, t = s[1] << 17;
        s[2] ^= s[0]; s[3] ^= s[1]; s[1] ^= s[2]; s[0] ^= s[3]; s[2] ^= t; s[3] = rotl(s[3], 45);
        return r;
    }
    double unif() { return (next() >> 11) * (1.0 / 9007199254740992.0); }
    uint64_t below(uint64_t n) { return n ? (uint64_t)(((unsigned __int128)next() * n) >> 64) : 0; }
    uint64_t geom(double mean) {                        // geometric on {1, 2, ...} with the given mean
        if (mean <= 1) return 1;
        const double p = 1.0 / mean;
        return 1 + (uint64_t)std::floor(std::log(1.0 - unif()) / std::log(1.0 - p));
    }
    uint64_t gap(double rate) {                         // bases until the next event of a per-base rate
        if (rate <= 0) return ~0ull >> 2;
        return (uint64_t)std::floor(std::log(1.0 - unif()) / std::log(1.0 - rate));
    }
    double normal() { const double u = std::max(unif(), 1e-300), v = unif(); return std::sqrt(-2 * std::log(u)) * std::cos(6.283185307179586 * v); }
};
const uint8_t ACGT[4] = {'A', 'C', 'G', 'T'};
struct CompLut {
    uint8_t t[256];
    CompLut() { for (int c = 0; c < 256; c++) t[c] = c == 'A' ? 'T' : c == 'C' ? 'G' : c == 'G' ? 'C' : c == 'T' ? 'A' : (uint8_t)c; }
};
const CompLut COMP;
inline uint8_t comp(uint8_t c) { return COMP.t[c]; }

void put_leb(std::vector<uint8_t>& o, uint64_t v) { while (v >= 0x80) { o.push_back((uint8_t)(v | 0x80)); v >>= 7; } o.push_back((uint8_t)v); }
void put32(std::vector<uint8_t>& o, uint32_t v) { o.insert(o.end(), (uint8_t*)&v, (uint8_t*)&v + 4); }
void put64(std::vector<uint8_t>& o, uint64_t v) { o.insert(o.end(), (uint8_t*)&v, (uint8_t*)&v + 8); }
uint64_t zz(int64_t v) { return ((uint64_t)v << 1) ^ (uint64_t)(v >> 63); }
// the decoder's bucket of a value (inverse of refrel3.h r3_unbucket): symbol, raw bit count, raw bits
uint32_t bucket(uint64_t v, uint32_t* nb, uint64_t* extra) {
    if (v < 16) { *nb = 0; *extra = 0; return (uint32_t)v; }
    const uint32_t e = 63 - __builtin_clzll(v);
    *nb = e - 2; *extra = v & ((1ull << (e - 2)) - 1);
    return 16 + (e - 4) * 4 + (uint32_t)((v >> (e - 2)) & 3);
}

// ---------------------------------------------------------------- the reference
struct Ref {
    std::vector<uint8_t> R;                        // upper-case bases (the decoded reference)
    std::vector<std::string> names; std::vector<uint64_t> lens, offs;
    std::vector<std::pair<uint64_t, uint64_t>> low; // soft-masked runs of its FASTA [start, end)
    uint8_t sha[32];
};

// ---------------------------------------------------------------- an assembly as pieces of its base stream
enum { PC_FWD = 0, PC_RC = 1, PC_LIT = 2 };
struct Piece { uint64_t at; uint64_t src; uint32_t len; uint32_t kind; };   // src: reference position or literal pool index

struct AsmSpec {
    uint64_t seed; uint32_t Q; double snv, indel, indel_mean; uint32_t indel_cap, n_sv, sv_min, sv_max;
    uint32_t ctg_min, ctg_max; double ctg_sigma, rc_frac, low_frac, low_mean, iupac; int block_hashes; int zlevel;
};

struct Asm {
    std::vector<Piece> pc; std::vector<uint8_t> lit;
    std::vector<std::string> hdr; std::vector<uint64_t> clen; std::vector<uint32_t> lw;
    std::vector<std::pair<uint64_t, uint64_t>> low; uint64_t n = 0;
};

void add_piece(std::vector<Piece>& v, uint64_t& at, uint32_t kind, uint64_t src, uint64_t len) {
    while (len) {
        const uint32_t l = (uint32_t)std::min<uint64_t>(len, 1u << 30);
        v.push_back({at, src, l, kind});
        at += l; len -= l;
        if (kind != PC_RC) src += l;
        else src += 0;                                      // a long reverse piece is split below by the caller
    }
}

// the mutated genome (all reference chromosomes in order) as pieces, then contigs, orientation, case
void make_assembly(const Ref& ref, const AsmSpec& S, Asm& A) {
    Rng g(S.seed);
    std::vector<Piece> gen; gen.reserve(1 << 20);
    std::vector<uint8_t>& lit = A.lit;
    uint64_t at = 0;
    for (size_t c = 0; c < ref.lens.size(); c++) {
        const uint64_t base = ref.offs[c], n = ref.lens[c];
        // structural variants of this chromosome: positions spread by length share
        std::vector<std::pair<uint64_t, int>> svs;
        const double share = (double)n / (double)ref.R.size();
        const uint64_t nsv = (uint64_t)std::floor(S.n_sv * share + g.unif());
        for (uint64_t k = 0; k < nsv; k++) svs.push_back({g.below(n), (int)g.below(3)});
        std::sort(svs.begin(), svs.end());
        size_t si = 0;
        uint64_t cur = 0, next_snv = g.gap(S.snv), next_ind = g.gap(S.indel);
        uint64_t run_start = 0;                          // start of the pending reference run
        auto flush_ref = [&](uint64_t end) { if (end > run_start) add_piece(gen, at, PC_FWD, base + run_start, end - run_start); };
        while (cur < n) {
            const uint64_t sv_at = si < svs.size() ? std::max(svs[si].first, cur) : n;
            const uint64_t e_snv = cur + next_snv, e_ind = cur + next_ind;
            const uint64_t ev = std::min(std::min(e_snv, e_ind), std::min(sv_at, n));
            if (ev >= n) { flush_ref(n); break; }
            if (ev == sv_at && si < svs.size()) {
                flush_ref(ev);
                const uint64_t L = std::min<uint64_t>(S.sv_min + g.below(S.sv_max - S.sv_min + 1), n - ev);
                const int kind = svs[si].second; si++;
                if (kind == 0) { cur = ev + L; }                                          // deletion
                else if (kind == 1) {                                                     // random insertion
                    const uint64_t p = lit.size();
                    for (uint64_t k = 0; k < L; k++) lit.push_back(ACGT[g.next() & 3]);
                    add_piece(gen, at, PC_LIT, p, L); cur = ev;
                } else {                                                                  // inversion
                    gen.push_back({at, base + ev, (uint32_t)L, PC_RC}); at += L; cur = ev + L;
                }
                run_start = cur;
                next_snv = g.gap(S.snv); next_ind = g.gap(S.indel);
                continue;
            }
            if (ev == e_snv) {
                const uint8_t r = ref.R[base + ev];
                const int k = r == 'A' ? 0 : r == 'C' ? 1 : r == 'G' ? 2 : r == 'T' ? 3 : -1;
                if (k >= 0) {
                    flush_ref(ev);
                    uint8_t alt = ACGT[(k + 1 + (int)g.below(3)) & 3];
                    if (S.iupac > 0 && g.unif() < S.iupac / S.snv) alt = (uint8_t)"RYKMSWBDHV"[g.below(10)];
                    lit.push_back(alt);
                    add_piece(gen, at, PC_LIT, lit.size() - 1, 1);
                    run_start = ev + 1;
                }
                cur = ev + 1;
                next_snv = g.gap(S.snv);
                next_ind = e_ind - cur;
                continue;
            }
            // indel
            flush_ref(ev);
            const uint64_t L = std::min<uint64_t>(g.geom(S.indel_mean), S.indel_cap);
            if (g.next() & 1) {
                const uint64_t p = lit.size();
                for (uint64_t k = 0; k < L; k++) lit.push_back(ACGT[g.next() & 3]);
                add_piece(gen, at, PC_LIT, p, L);
                cur = ev;
            } else {
                cur = std::min(n, ev + L);
            }
            run_start = cur;
            next_ind = g.gap(S.indel);
            next_snv = e_snv > cur ? e_snv - cur : 0;
        }
    }
    const uint64_t total = at;
    A.n = total;
    // contigs: lognormal lengths scaled to the total
    const uint32_t nctg = (uint32_t)std::max<uint64_t>(1, std::min<uint64_t>(total, S.ctg_min + g.below(S.ctg_max - S.ctg_min + 1)));
    std::vector<double> w(nctg);
    double sw = 0;
    for (auto& x : w) { x = std::exp(S.ctg_sigma * g.normal()); sw += x; }
    std::vector<uint64_t> cut(nctg + 1, 0);
    for (uint32_t k = 0; k < nctg; k++) cut[k + 1] = cut[k] + std::max<uint64_t>(1, (uint64_t)(w[k] / sw * (double)total));
    cut[nctg] = total;
    for (uint32_t k = nctg - 1; k > 0 && cut[k] >= cut[k + 1]; k--) cut[k] = cut[k + 1] - 1;
    // assemble the stream contig by contig (a reverse-complemented contig reverses its pieces and flips each)
    std::vector<Piece>& out = A.pc; out.reserve(gen.size() + 2 * nctg);
    size_t pi = 0; uint64_t oat = 0;
    for (uint32_t k = 0; k < nctg; k++) {
        const uint64_t c0 = cut[k], c1 = cut[k + 1];
        const bool rc = g.unif() < S.rc_frac;
        std::vector<Piece> seg;
        while (pi < gen.size() && gen[pi].at + gen[pi].len <= c0) pi++;
        for (size_t q = pi; q < gen.size() && gen[q].at < c1; q++) {
            Piece p = gen[q];
            const uint64_t a = std::max(p.at, c0), e = std::min<uint64_t>(p.at + p.len, c1);
            if (a >= e) continue;
            const uint64_t skip = a - p.at, len = e - a;
            Piece s{a - c0, 0, (uint32_t)len, p.kind};
            if (p.kind == PC_FWD || p.kind == PC_LIT) s.src = p.src + skip;
            else s.src = p.src + (p.len - skip - len);                 // reverse piece: its tail reference span
            seg.push_back(s);
        }
        const uint64_t L = c1 - c0;
        if (rc) {
            std::reverse(seg.begin(), seg.end());
            for (auto& s : seg) {
                s.at = L - (s.at + s.len);
                if (s.kind == PC_FWD) s.kind = PC_RC;
                else if (s.kind == PC_RC) s.kind = PC_FWD;
                else {                                                // literals: complemented, reversed, new pool entry
                    const uint64_t p = lit.size();
                    for (uint32_t i = 0; i < s.len; i++) lit.push_back(comp(lit[s.src + s.len - 1 - i]));
                    s.src = p;
                }
            }
        }
        for (auto& s : seg) { s.at += oat; out.push_back(s); }
        char h[96];
        snprintf(h, sizeof h, "ctg%u%s len=%llu", k + 1, rc ? " rc" : "", (unsigned long long)L);
        A.hdr.push_back(h); A.clen.push_back(L); A.lw.push_back(k % 2 ? 80 : 60);
        oat += L;
    }
    // soft-masked runs over the stream
    if (S.low_frac > 0) {
        const double gap_mean = S.low_mean / S.low_frac - S.low_mean;
        uint64_t x = g.geom(gap_mean);
        while (x < total) {
            const uint64_t l = std::min<uint64_t>(g.geom(S.low_mean), total - x);
            A.low.push_back({x, x + l});
            x += l + g.geom(gap_mean);
        }
    }
}

// upper-case bases of stream [a, a + n) into out
void materialize(const Ref& ref, const Asm& A, size_t& pi, uint64_t a, uint64_t n, uint8_t* out) {
    while (pi > 0 && A.pc[pi].at > a) pi--;
    while (pi < A.pc.size() && A.pc[pi].at + A.pc[pi].len <= a) pi++;
    for (size_t q = pi; q < A.pc.size() && A.pc[q].at < a + n; q++) {
        const Piece& p = A.pc[q];
        const uint64_t x0 = std::max(p.at, a), x1 = std::min<uint64_t>(p.at + p.len, a + n);
        const uint64_t k = x0 - p.at;
        uint8_t* o = out + (x0 - a);
        if (p.kind == PC_FWD) memcpy(o, &ref.R[p.src + k], x1 - x0);
        else if (p.kind == PC_LIT) memcpy(o, &A.lit[p.src + k], x1 - x0);
        else { const uint8_t* top = &ref.R[p.src + p.len - 1 - k]; for (uint64_t i = 0, n2 = x1 - x0; i < n2; i++) o[i] = COMP.t[*(top - i)]; }
    }
}
// one upper-case base of the stream (the literal bytes of the counting pass)
uint8_t base_at(const Ref& ref, const Asm& A, size_t q, uint64_t x) {
    while (q + 1 < A.pc.size() && A.pc[q].at + A.pc[q].len <= x) q++;
    while (q > 0 && A.pc[q].at > x) q--;
    const Piece& p = A.pc[q];
    const uint64_t k = x - p.at;
    if (p.kind == PC_FWD) return ref.R[p.src + k];
    if (p.kind == PC_LIT) return A.lit[p.src + k];
    return COMP.t[ref.R[p.src + p.len - 1 - k]];
}

// ---------------------------------------------------------------- events -> symbols (the decoder's order and contexts)
struct Sym { uint8_t ctx; uint8_t raw; uint8_t nb; uint8_t pad; uint32_t v; };  // raw: v holds nb raw bits (<= 16)
struct Diag { int64_t c; uint32_t dir; };

struct BlockCoder {
    const Ref& ref; const Asm& A; uint32_t Q;
    std::vector<Sym> syms; std::vector<uint8_t> bases;
    BlockCoder(const Ref& r, const Asm& a, uint32_t q) : ref(r), A(a), Q(q) { bases.resize(q); }

    static int kcls(int k) { return k < 0 ? 0 : k == K_CONT ? 1 : (k == K_DELTA || k == K_REP || k == K_FLIP) ? 2 : 3; }
    static int llcl(uint64_t ll) { return ll == 0 ? 0 : ll == 1 ? 1 : ll <= 8 ? 2 : 3; }
    void sym(int ctx, uint32_t s) { syms.push_back({(uint8_t)ctx, 0, 0, 0, s}); }
    void raw(uint32_t nb, uint64_t v) {                     // decoder order: the low 16 bits first
        while (nb) { const uint32_t k = nb > 16 ? 16 : nb; syms.push_back({0, 1, (uint8_t)k, 0, (uint32_t)(v & ((1u << k) - 1))}); v >>= k; nb -= k; }
    }
    void val(int ctx, uint64_t v) { uint32_t nb; uint64_t ex; const uint32_t s = bucket(v, &nb, &ex); sym(ctx, s); raw(nb, ex); }
    int refbase(const Diag& g, uint32_t o) const {
        const int64_t q = g.dir ? g.c - (int64_t)o : g.c + (int64_t)o;
        if (q < 0 || (uint64_t)q >= ref.R.size()) return 4;
        const uint8_t b = g.dir ? comp(ref.R[q]) : ref.R[q];
        return b == 'A' ? 0 : b == 'C' ? 1 : b == 'G' ? 2 : b == 'T' ? 3 : 4;
    }
    static void push(Diag* cache, int& nc, Diag g) {
        int j = 0;
        while (j < nc && !(cache[j].c == g.c && cache[j].dir == g.dir)) j++;
        if (j == nc) { if (nc < 4) nc++; j = nc - 1; }
        for (; j > 0; j--) cache[j] = cache[j - 1];
        cache[0] = g;
    }
    static Diag diag_of(uint32_t dir, uint64_t p, uint32_t o, uint64_t L) {
        return dir ? Diag{(int64_t)p + (int64_t)L - 1 + (int64_t)o, 1} : Diag{(int64_t)p - (int64_t)o, 0};
    }
    // symbols of block b; st = the block's start diagonal. Literal bytes come from `bases` when the block was
    // materialized there, else straight from the pieces.
    void code(uint64_t b, size_t& pi, Diag st, bool materialized) {
        syms.clear();
        const uint64_t bst = b * Q, blen = std::min<uint64_t>(Q, A.n - bst);
        while (pi > 0 && A.pc[pi].at > bst) pi--;
        while (pi < A.pc.size() && A.pc[pi].at + A.pc[pi].len <= bst) pi++;
        const size_t pi0 = pi;
        Diag cache[4]; int nc = 1; cache[0] = st; int prevk = -1;
        uint32_t o = 0;
        auto literals = [&](uint32_t upto) {                // the run [o, upto), then its LL context is already given
            const uint64_t ll = upto - o;
            val(C_LL + kcls(prevk), ll);
            uint32_t p1 = 16, p2 = 16;
            for (uint32_t j = 0; j < ll; j++) {
                const uint8_t by = materialized ? bases[o + j] : base_at(ref, A, pi0, bst + o + j);
                int c;
                if (ll <= 8) c = C_LITR + refbase(cache[0], o + j) * 2 + (j == 0 ? 1 : 0);
                else c = C_LIT2 + (p1 == 16 ? 16 : (int)((p2 == 16 ? p1 : p2 * 4 + p1) % 16));
                const uint32_t s = by == 'A' ? 0 : by == 'C' ? 1 : by == 'G' ? 2 : by == 'T' ? 3 : by == 'N' ? 4 : 5;
                sym(c, s);
                if (s == 5) raw(8, by);
                p2 = p1; p1 = s < 4 ? s : 0;
            }
            o = upto;
            return ll;
        };
        size_t q = pi;
        uint32_t lit_from = 0;                              // literal run start (bases not covered by a copy yet)
        while (true) {
            // next copy: a reference segment of >= 12 bases inside the block
            uint32_t c_at = (uint32_t)blen, c_len = 0, c_dir = 0; uint64_t c_p = 0;
            for (; q < A.pc.size() && A.pc[q].at < bst + blen; q++) {
                const Piece& p = A.pc[q];
                const uint64_t x0 = std::max(p.at, bst + o), x1 = std::min<uint64_t>(p.at + p.len, bst + blen);
                if (x0 >= x1 || p.kind == PC_LIT || x1 - x0 < MINL) continue;
                const uint64_t k = x0 - p.at;
                c_at = (uint32_t)(x0 - bst); c_len = (uint32_t)(x1 - x0); c_dir = p.kind == PC_RC;
                c_p = p.kind == PC_FWD ? p.src + k : p.src + p.len - k - (x1 - x0);
                break;
            }
            (void)lit_from;
            const uint64_t ll = literals(c_at);
            if (o == blen) break;
            // the copy's kind against the diagonal cache (cheapest of continue / delta / recent / other strand / absolute)
            int kind = K_ABS, ki = 0; uint64_t z = 0; double best = 1e9;
            for (int k = 0; k < nc; k++) {
                const bool same = (uint32_t)cache[k].dir == c_dir;
                int64_t d;
                if (same) d = (int64_t)c_p - (cache[k].dir ? cache[k].c - (int64_t)o - (int64_t)c_len + 1 : cache[k].c + (int64_t)o);
                else d = (int64_t)c_p - (cache[k].dir ? cache[k].c - (int64_t)o : cache[k].c + (int64_t)o);
                const uint64_t a = (uint64_t)(d < 0 ? -d : d);
                if (a >= (1ull << 24)) continue;
                if (!same && k >= nc) continue;
                if (same && k == 0 && d == 0) { if (0 < best) { best = 0; kind = K_CONT; ki = 0; z = 0; } continue; }
                const double cost = (a ? 64 - __builtin_clzll(a) : 0) + 6.0 + (k || !same ? 2.0 : 0.0);
                if (cost < best && !(same && k > 0 && k >= nc)) {
                    best = cost; kind = !same ? K_FLIP : k == 0 ? K_DELTA : K_REP; ki = k; z = zz(d);
                }
            }
            if (kind == K_ABS && c_p >= (1ull << 32)) kind = K_ABS;   // references are < 2^32 bases (checked at open)
            sym(C_KIND + llcl(ll) * 4 + kcls(prevk), (uint32_t)kind);
            if (kind == K_DELTA) val(C_DELTA + (ll == 0 ? 0 : 1), z);
            else if (kind == K_REP) { sym(C_REPK, (uint32_t)(ki - 1)); val(C_REPD, z); }
            else if (kind == K_ABS) { sym(C_DIR, c_dir); raw(32, c_p); }
            else if (kind == K_FLIP) { sym(C_FLIPK, (uint32_t)ki); val(C_FLIPD, z); }
            val(C_LEN + kind, c_len - MINL);
            push(cache, nc, diag_of(c_dir, c_p, o, c_len));
            o += c_len; prevk = kind;
            if (o == blen) break;
            if (q < A.pc.size() && A.pc[q].at + A.pc[q].len <= bst + o) q++;
        }
    }
};

// normalise counts to frequencies summing to 4096, every seen symbol at least 1
void normalise(const uint64_t* cnt, int n, uint16_t* f) {
    uint64_t tot = 0;
    for (int s = 0; s < n; s++) tot += cnt[s];
    for (int s = 0; s < n; s++) f[s] = 0;
    if (!tot) return;
    int64_t sum = 0; int big = 0;
    for (int s = 0; s < n; s++) {
        if (!cnt[s]) continue;
        uint64_t v = (uint64_t)((double)cnt[s] * MTOT / (double)tot);
        if (!v) v = 1;
        f[s] = (uint16_t)v; sum += v;
        if (cnt[s] > cnt[big]) big = s;
    }
    while (sum > (int64_t)MTOT) {                           // take from the largest frequencies
        int b = -1;
        for (int s = 0; s < n; s++) if (f[s] > 1 && (b < 0 || f[s] > f[b])) b = s;
        const int64_t take = std::min<int64_t>(sum - MTOT, f[b] - 1);
        f[b] = (uint16_t)(f[b] - take); sum -= take;
    }
    if (sum < (int64_t)MTOT) f[big] = (uint16_t)(f[big] + (MTOT - sum));
}

// byte-wise rANS, backwards from 2^16; the stream starts with the final state's 3 bytes (refrel3.h r3_dinit)
void rans_encode(const std::vector<Sym>& syms, const uint16_t* freq, const uint16_t* cum, std::vector<uint8_t>& out) {
    std::vector<uint8_t> rev; rev.reserve(syms.size() + 16);
    uint32_t x = RANS_L;
    for (size_t i = syms.size(); i-- > 0;) {
        const Sym& s = syms[i];
        if (s.raw) {
            const uint32_t xmax = (RANS_L >> s.nb) << 8;
            while (x >= xmax) { rev.push_back((uint8_t)x); x >>= 8; }
            x = (x << s.nb) | s.v;
        } else {
            const uint32_t f = freq[s.ctx * AB + s.v], c = cum[s.ctx * (AB + 1) + s.v];
            const uint32_t xmax = ((RANS_L >> PB) << 8) * f;
            while (x >= xmax) { rev.push_back((uint8_t)x); x >>= 8; }
            x = ((x / f) << PB) + (x % f) + c;
        }
    }
    out.push_back((uint8_t)x); out.push_back((uint8_t)(x >> 8)); out.push_back((uint8_t)(x >> 16));
    out.insert(out.end(), rev.rbegin(), rev.rend());
}

struct Hasher {
    XXH3_state_t* h;
    Hasher() : h(XXH3_createState()) { XXH3_64bits_reset(h); }
    ~Hasher() { XXH3_freeState(h); }
    void add(const void* p, size_t n) { XXH3_64bits_update(h, p, n); }
    uint64_t digest() const { return XXH3_64bits_digest(h); }
};

// one archive: pieces -> two passes over the blocks (count, then encode) with the stream hashed alongside
std::vector<uint8_t> encode_archive(const Ref& ref, const Asm& A, const AsmSpec& S, const std::string& refname, FILE* fasta_out) {
    const uint32_t Q = S.Q;
    const uint64_t nb = (A.n + Q - 1) / Q;
    std::vector<uint64_t> cnt((size_t)NCTX * AB, 0);
    std::vector<Diag> st(nb);
    BlockCoder bc(ref, A, Q);
    // start diagonal of each block: the reference segment covering its first base if any, else the carried one
    {
        Diag carry{0, 0};
        size_t pi = 0;
        for (uint64_t b = 0; b < nb; b++) {
            const uint64_t bst = b * Q;
            while (pi < A.pc.size() && A.pc[pi].at + A.pc[pi].len <= bst) pi++;
            Diag g = b == 0 ? Diag{0, 0} : Diag{carry.dir ? carry.c - (int64_t)Q : carry.c + (int64_t)Q, carry.dir};
            for (size_t q = pi; q < A.pc.size() && A.pc[q].at < bst + Q; q++) {
                const Piece& p = A.pc[q];
                if (p.kind == PC_LIT) continue;
                const uint64_t x0 = std::max(p.at, bst), k = x0 - p.at;
                const uint32_t o = (uint32_t)(x0 - bst);
                if (p.kind == PC_FWD) g = Diag{(int64_t)(p.src + k) - (int64_t)o, 0};
                else g = Diag{(int64_t)(p.src + p.len - 1 - k) + (int64_t)o, 1};
                break;
            }
            st[b] = g; carry = g;
        }
    }
    size_t pi = 0;
    for (uint64_t b = 0; b < nb; b++) {
        bc.code(b, pi, st[b], false);
        for (auto& s : bc.syms) if (!s.raw) cnt[(size_t)s.ctx * AB + s.v]++;
    }
    std::vector<uint16_t> freq((size_t)NCTX * AB, 0), cum((size_t)NCTX * (AB + 1), 0);
    for (int c = 0; c < NCTX; c++) {
        normalise(&cnt[(size_t)c * AB], alpha(c), &freq[(size_t)c * AB]);
        uint32_t a = 0;
        for (int s = 0; s < AB; s++) { cum[(size_t)c * (AB + 1) + s] = (uint16_t)a; a += freq[(size_t)c * AB + s]; }
        cum[(size_t)c * (AB + 1) + AB] = (uint16_t)a;
    }
    std::vector<uint8_t> payload; payload.reserve(nb * 64);
    std::vector<uint64_t> plen(nb), bhash(S.block_hashes ? nb : 0);
    Hasher hb, hf;                                            // base stream (case kept) and FASTA file hashes
    std::vector<uint8_t> cased(Q), fa; fa.reserve((size_t)Q * 2 + 4096);
    size_t lowi = 0, ctg = 0; uint64_t in_ctg = 0;            // FASTA layout state
    pi = 0;
    for (uint64_t b = 0; b < nb; b++) {
        const uint64_t bst = b * Q, blen = std::min<uint64_t>(Q, A.n - bst);
        size_t mp = pi;
        materialize(ref, A, mp, bst, blen, bc.bases.data());
        bc.code(b, pi, st[b], true);
        const size_t at = payload.size();
        rans_encode(bc.syms, freq.data(), cum.data(), payload);
        plen[b] = payload.size() - at;
        if (S.block_hashes) bhash[b] = XXH3_64bits(bc.bases.data(), blen);
        memcpy(cased.data(), bc.bases.data(), blen);
        while (lowi < A.low.size() && A.low[lowi].second <= bst) lowi++;
        for (size_t r = lowi; r < A.low.size() && A.low[r].first < bst + blen; r++) {
            const uint64_t x0 = std::max(A.low[r].first, bst), x1 = std::min(A.low[r].second, bst + blen);
            for (uint64_t x = x0; x < x1; x++) cased[x - bst] |= 0x20;
        }
        hb.add(cased.data(), blen);
        fa.clear();
        uint64_t done = 0;
        while (done < blen) {
            while (ctg < A.clen.size() && in_ctg == A.clen[ctg]) { ctg++; in_ctg = 0; }
            if (in_ctg == 0) { fa.push_back('>'); fa.insert(fa.end(), A.hdr[ctg].begin(), A.hdr[ctg].end()); fa.push_back('\n'); }
            const uint64_t lw = A.lw[ctg], room = lw - in_ctg % lw;
            const uint64_t k = std::min(std::min(room, A.clen[ctg] - in_ctg), blen - done);
            fa.insert(fa.end(), cased.data() + done, cased.data() + done + k);
            done += k; in_ctg += k;
            if (in_ctg % lw == 0 || in_ctg == A.clen[ctg]) fa.push_back('\n');
        }
        hf.add(fa.data(), fa.size());
        if (fasta_out) fwrite(fa.data(), 1, fa.size(), fasta_out);
    }
    // contigs of length 0 at the end (none are made; kept for the layout's completeness)
    // meta
    std::vector<uint8_t> M;
    put32(M, (uint32_t)A.hdr.size());
    for (size_t r = 0; r < A.hdr.size(); r++) { put32(M, (uint32_t)A.hdr[r].size()); M.insert(M.end(), A.hdr[r].begin(), A.hdr[r].end()); put64(M, A.clen[r]); put32(M, A.lw[r]); }
    put64(M, A.low.size());
    uint64_t last = 0;
    for (auto& r : A.low) { put_leb(M, r.first - last); put_leb(M, r.second - r.first); last = r.second; }
    for (int c = 0; c < NCTX; c++) for (int s = 0; s < alpha(c); s++) put_leb(M, freq[(size_t)c * AB + s]);
    uint64_t prevc = 0; uint32_t prevd = 0;
    for (uint64_t b = 0; b < nb; b++) {
        put_leb(M, plen[b]);
        const int64_t pred = b == 0 ? 0 : (int64_t)(prevd ? prevc - Q : prevc + Q);
        put_leb(M, zz(st[b].c - pred) * 2 + st[b].dir);
        prevc = (uint64_t)st[b].c; prevd = st[b].dir;
    }
    std::vector<uint8_t> MZ(ZSTD_compressBound(M.size()));
    const size_t mz = ZSTD_compress(MZ.data(), MZ.size(), M.data(), M.size(), S.zlevel);
    if (ZSTD_isError(mz)) throw std::runtime_error("zstd");
    MZ.resize(mz);
    std::vector<uint8_t> o(136, 0);
    memcpy(&o[0], "RFRL3V1\0", 8);
    auto p32 = [&](size_t at, uint32_t v) { memcpy(&o[at], &v, 4); };
    auto p64 = [&](size_t at, uint64_t v) { memcpy(&o[at], &v, 8); };
    p32(8, 1); p32(12, Q); p32(16, S.block_hashes ? 1 : 0); p32(20, 0);
    memcpy(&o[24], ref.sha, 32); p64(56, ref.R.size()); p64(64, A.n); p64(72, nb); p64(80, hf.digest()); p64(88, hb.digest());
    p64(96, MZ.size()); p64(104, M.size()); p64(112, S.block_hashes ? nb * 8 : 0); p64(120, payload.size());
    const uint16_t nl = (uint16_t)std::min<size_t>(refname.size(), 65535);
    o.push_back((uint8_t)nl); o.push_back((uint8_t)(nl >> 8));
    o.insert(o.end(), refname.begin(), refname.begin() + nl);
    o.insert(o.end(), MZ.begin(), MZ.end());
    for (uint64_t b = 0; b < (S.block_hashes ? nb : 0); b++) put64(o, bhash[b]);
    const uint64_t hx = XXH3_64bits(o.data(), o.size());
    p64(128, hx);
    o.insert(o.end(), payload.begin(), payload.end());
    return o;
}

}  // namespace

extern "C" {

struct pvs_ref;
const char* pvs_last_error(void) { return g_err.c_str(); }

// a reference of `n` contigs with the given lengths: uniform ACGT, N runs of n_run bases covering n_frac, soft-masked
// runs (geometric, mean low_mean) covering low_frac of its FASTA
pvs_ref* pvs_ref_generate(uint64_t seed, const uint64_t* lens, int n, double n_frac, uint64_t n_run, double low_frac, double low_mean,
                          int threads) {
    Ref* r = new Ref();
    uint64_t tot = 0;
    for (int i = 0; i < n; i++) { r->offs.push_back(tot); r->lens.push_back(lens[i]); tot += lens[i]; char h[32]; snprintf(h, sizeof h, "chr%d", i + 1); r->names.push_back(h); }
    r->R.resize(tot);
    const uint64_t chunk = 1 << 22, nch = (tot + chunk - 1) / chunk;
    std::atomic<uint64_t> next{0};
    std::vector<std::thread> th;
    for (int t = 0; t < std::max(1, threads); t++) th.emplace_back([&] {
        for (;;) {
            const uint64_t c = next.fetch_add(1);
            if (c >= nch) break;
            Rng g(seed ^ (0xA5A5A5A5ull + c * 0x9E3779B97F4A7C15ull));
            const uint64_t a = c * chunk, e = std::min(tot, a + chunk);
            for (uint64_t i = a; i < e;) { uint64_t v = g.next(); for (int k = 0; k < 32 && i < e; k++, i++, v >>= 2) r->R[i] = ACGT[v & 3]; }
        }
    });
    for (auto& x : th) x.join();
    Rng g(seed * 31 + 7);
    for (int i = 0; i < n; i++) {
        const uint64_t runs = (uint64_t)std::floor(n_frac * (double)lens[i] / (double)std::max<uint64_t>(1, n_run) + g.unif());
        for (uint64_t k = 0; k < runs && lens[i] > n_run; k++) { const uint64_t p = r->offs[i] + g.below(lens[i] - n_run); memset(&r->R[p], 'N', n_run); }
        if (low_frac > 0) {
            const double gm = low_mean / low_frac - low_mean;
            uint64_t x = g.geom(gm);
            while (x < lens[i]) { const uint64_t l = std::min<uint64_t>(g.geom(low_mean), lens[i] - x); r->low.push_back({r->offs[i] + x, r->offs[i] + x + l}); x += l + g.geom(gm); }
        }
    }
    SHA256(r->R.data(), r->R.size(), r->sha);
    return (pvs_ref*)r;
}

void pvs_ref_free(pvs_ref* r) { delete (Ref*)r; }
uint64_t pvs_ref_n(const pvs_ref* r) { return ((const Ref*)r)->R.size(); }
void pvs_ref_sha256(const pvs_ref* r, uint8_t out[32]) { memcpy(out, ((const Ref*)r)->sha, 32); }

// the reference FASTA: headers chrN, line width lw, soft-masked runs in lower case
int pvs_ref_write_fasta(const pvs_ref* rp, const char* path, uint32_t lw) {
    const Ref& r = *(const Ref*)rp;
    FILE* f = fopen(path, "wb");
    if (!f) { g_err = std::string(path) + ": cannot write"; return 1; }
    std::vector<uint8_t> buf; buf.reserve(1 << 22);
    size_t li = 0;
    for (size_t i = 0; i < r.lens.size(); i++) {
        buf.push_back('>'); buf.insert(buf.end(), r.names[i].begin(), r.names[i].end()); buf.push_back('\n');
        for (uint64_t x = 0; x < r.lens[i]; x += lw) {
            const uint64_t k = std::min<uint64_t>(lw, r.lens[i] - x), a = r.offs[i] + x;
            const size_t at = buf.size();
            buf.insert(buf.end(), &r.R[a], &r.R[a] + k);
            while (li < r.low.size() && r.low[li].second <= a) li++;
            for (size_t q = li; q < r.low.size() && r.low[q].first < a + k; q++)
                for (uint64_t y = std::max(r.low[q].first, a); y < std::min(r.low[q].second, a + k); y++) buf[at + (y - a)] |= 0x20;
            buf.push_back('\n');
            if (buf.size() > (1u << 22)) { fwrite(buf.data(), 1, buf.size(), f); buf.clear(); }
        }
    }
    fwrite(buf.data(), 1, buf.size(), f);
    const int bad = fclose(f) != 0;
    if (bad) g_err = std::string(path) + ": write failed";
    return bad;
}

struct pvs_spec {
    uint64_t seed; uint32_t Q; double snv, indel, indel_mean; uint32_t indel_cap, n_sv, sv_min, sv_max;
    uint32_t ctg_min, ctg_max; double ctg_sigma, rc_frac, low_frac, low_mean, iupac; int32_t block_hashes, zlevel;
};

// one archive per spec written to paths[i] (fasta_paths[i] != NULL also writes the assembly FASTA), on `threads`
// host threads; 0 or the first failure (pvs_last_error)
int pvs_make_archives(const pvs_ref* rp, const pvs_spec* specs, int n, const char* const* paths, const char* const* fasta_paths,
                      const char* refname, int threads) {
    const Ref& ref = *(const Ref*)rp;
    std::atomic<int> next{0};
    std::mutex mu; std::string first;
    std::vector<std::thread> th;
    for (int t = 0; t < std::max(1, std::min(threads, n)); t++) th.emplace_back([&] {
        for (;;) {
            const int i = next.fetch_add(1);
            if (i >= n) break;
            try {
                const pvs_spec& s = specs[i];
                AsmSpec S{s.seed, s.Q, s.snv, s.indel, s.indel_mean, s.indel_cap, s.n_sv, s.sv_min, s.sv_max, s.ctg_min, s.ctg_max,
                          s.ctg_sigma, s.rc_frac, s.low_frac, s.low_mean, s.iupac, s.block_hashes, s.zlevel};
                Asm A;
                make_assembly(ref, S, A);
                FILE* ff = fasta_paths && fasta_paths[i] ? fopen(fasta_paths[i], "wb") : nullptr;
                const std::vector<uint8_t> arc = encode_archive(ref, A, S, refname, ff);
                if (ff) fclose(ff);
                FILE* f = fopen(paths[i], "wb");
                if (!f || fwrite(arc.data(), 1, arc.size(), f) != arc.size()) throw std::runtime_error(std::string(paths[i]) + ": write failed");
                fclose(f);
            } catch (const std::exception& e) {
                std::lock_guard<std::mutex> g(mu);
                if (first.empty()) first = e.what();
            }
        }
    });
    for (auto& x : th) x.join();
    if (!first.empty()) { g_err = first; return 1; }
    return 0;
}

}  // extern "C"
