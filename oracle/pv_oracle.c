/* pv_oracle.c - TEST INFRASTRUCTURE ONLY (the parity checker; see pv_oracle.h). A plain-C restatement of the
 * reference's refrel3 v1 reader and CPU decoder, panvram 1.0.1. Every function cites the reference lines it follows.
 * Third-party arithmetic comes from the image's own runtime libraries: XXH3_64bits (xxHash 0.8, libxxhash.so.0),
 * ZSTD_decompress (libzstd.so.1) and SHA-256 (OpenSSL libcrypto.so.3). */
#define _GNU_SOURCE
#include "pv_oracle.h"

#include <openssl/sha.h>
#include <pthread.h>
#include <stdatomic.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

/* ---- runtime-library prototypes (the image has the shared objects, not their headers) ---- */
unsigned long long ZSTD_getFrameContentSize(const void* src, size_t srcSize);
size_t ZSTD_findFrameCompressedSize(const void* src, size_t srcSize);
size_t ZSTD_decompress(void* dst, size_t dstCapacity, const void* src, size_t compressedSize);
uint64_t XXH3_64bits(const void* data, size_t len);
typedef struct XXH3_state_s XXH3_state_t;
XXH3_state_t* XXH3_createState(void);
int XXH3_freeState(XXH3_state_t* s);
int XXH3_64bits_reset(XXH3_state_t* s);
int XXH3_64bits_update(XXH3_state_t* s, const void* p, size_t n);
uint64_t XXH3_64bits_digest(const XXH3_state_t* s);

/* ---- the refrel3 model: contexts, kinds, alphabets (refrel3.h:24-43) ---- */
enum { C_LL = 0, C_LITR = 4, C_LIT2 = 14, C_KIND = 31, C_DELTA = 47, C_REPK = 49, C_REPD = 50, C_DIR = 51, C_SELF = 52,
       C_LEN = 53, C_FLIPK = 59, C_FLIPD = 60, NCTX = 61 };
enum { K_CONT = 0, K_DELTA = 1, K_REP = 2, K_ABS = 3, K_SELF = 4, K_FLIP = 5 };
#define AB 104
#define PB 12u
#define MTOT (1u << PB)
#define RL (1u << 16)
#define MINL 12u
#define MAXOPS 4096u
static int alpha_of(int c) {
    if (c < C_LITR) return AB;                      /* LL x previous kind class */
    if (c < C_DELTA) return 6;                      /* LITR, LIT2, KIND */
    if (c < C_REPK) return AB;                      /* DELTA */
    if (c == C_REPK) return 3;
    if (c == C_REPD) return AB;
    if (c == C_DIR) return 2;
    if (c == C_SELF) return AB;
    if (c < C_FLIPK) return AB;                     /* LEN x kind */
    if (c == C_FLIPK) return 4;
    return AB;                                      /* FLIP delta */
}

typedef struct { uint16_t freq[NCTX][AB]; uint16_t cum[NCTX][AB + 1]; uint8_t sym[NCTX][MTOT]; } tab_t;  /* R3Tab */

/* refrel3.h:55-63 */
static uint64_t unbucket(uint32_t s, uint64_t extra) {
    if (s < 16) return s;
    const uint32_t e = (s - 16) / 4 + 4, m = (s - 16) & 3;
    return (1ull << e) | ((uint64_t)m << (e - 2)) | extra;
}
static uint32_t nbits(uint32_t s) { return s < 16 ? 0 : (s - 16) / 4 + 2; }
static int llc(uint64_t ll) { return ll == 0 ? 0 : ll == 1 ? 1 : ll <= 8 ? 2 : 3; }
static int kclass(int k) { return k < 0 ? 0 : k == K_CONT ? 1 : (k == K_DELTA || k == K_REP || k == K_FLIP) ? 2 : 3; }
static int b2(uint8_t c) { switch (c) { case 'A': return 0; case 'C': return 1; case 'G': return 2; case 'T': return 3; case 'N': return 4; default: return 5; } }
/* refrel_format.h:75 - complement of upper-case ACGT, every other byte unchanged */
static uint8_t comp_up(uint8_t c) { switch (c) { case 'A': return 'T'; case 'C': return 'G'; case 'G': return 'C'; case 'T': return 'A'; default: return c; } }
/* pv_v1.h:74-76 - complement keeping case; token map */
static uint8_t comp_case(uint8_t c) {
    switch (c) { case 'A': return 'T'; case 'C': return 'G'; case 'G': return 'C'; case 'T': return 'A';
                 case 'a': return 't'; case 'c': return 'g'; case 'g': return 'c'; case 't': return 'a'; default: return c; }
}
static uint8_t token(uint8_t c) { switch (c | 0x20) { case 'a': return 0; case 'c': return 1; case 'g': return 2; case 't': return 3; default: return 4; } }

/* pv_v1.h:56-58 (build_tab) */
static void build_tab(tab_t* T) {
    for (int c = 0; c < NCTX; c++) {
        uint32_t a = 0;
        for (int s = 0; s < AB; s++) {
            T->cum[c][s] = (uint16_t)a;
            for (uint32_t k = 0; k < T->freq[c][s]; k++) T->sym[c][a + k] = (uint8_t)s;
            a += T->freq[c][s];
        }
        T->cum[c][AB] = (uint16_t)a;
    }
}

/* ---- rANS, byte-wise, state in [2^16, 2^24) (refrel3.h:69-91) ---- */
typedef struct { const uint8_t* p; const uint8_t* e; uint32_t x; int bad; } rdec;
static void rd_init(rdec* d, const uint8_t* p, uint32_t n) {
    d->p = p; d->e = p + n; d->bad = 0; d->x = 0;
    if (n < 3) { d->bad = 1; return; }
    d->x = (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16);
    d->p += 3;
}
static uint32_t rd_sym(rdec* d, const tab_t* T, int c) {
    const uint32_t slot = d->x & (MTOT - 1), s = T->sym[c][slot], f = T->freq[c][s];
    if (!f) { d->bad = 1; return 0; }
    d->x = f * (d->x >> PB) + slot - T->cum[c][s];
    while (d->x < RL) { if (d->p >= d->e) { d->bad = 1; return s; } d->x = (d->x << 8) | *d->p++; }
    return s;
}
static uint64_t rd_raw(rdec* d, uint32_t nb) {
    uint64_t v = 0; uint32_t sh = 0;
    while (nb) {
        const uint32_t k = nb > 16 ? 16 : nb, b = d->x & ((1u << k) - 1);
        d->x >>= k;
        while (d->x < RL) { if (d->p >= d->e) { d->bad = 1; return v; } d->x = (d->x << 8) | *d->p++; }
        v |= (uint64_t)b << sh; sh += k; nb -= k;
    }
    return v;
}
static uint64_t rd_val(rdec* d, const tab_t* T, int c) { const uint32_t s = rd_sym(d, T, c); return unbucket(s, rd_raw(d, nbits(s))); }
static int64_t unzz(uint64_t z) { return (int64_t)(z >> 1) ^ -(int64_t)(z & 1); }

/* ---- diagonals and their cache (refrel3.h:94-102) ---- */
typedef struct { uint64_t c; uint32_t dir; } diag_t;
static int64_t dexp(diag_t g, uint32_t o, uint64_t L) { return g.dir ? (int64_t)g.c - (int64_t)o - (int64_t)L + 1 : (int64_t)g.c + (int64_t)o; }
static int64_t dlocus(diag_t g, uint32_t o) { return g.dir ? (int64_t)g.c - (int64_t)o : (int64_t)g.c + (int64_t)o; }
static diag_t dmake(uint32_t dir, uint64_t p, uint32_t o, uint64_t L) {
    diag_t g; g.dir = dir;
    g.c = dir ? (uint64_t)((int64_t)p + (int64_t)L - 1 + (int64_t)o) : (uint64_t)((int64_t)p - (int64_t)o);
    return g;
}
static void dpush(diag_t* cache, int* nc, diag_t g) {
    int j = 0;
    while (j < *nc && !(cache[j].c == g.c && cache[j].dir == g.dir)) j++;
    if (j == *nc) { if (*nc < 4) (*nc)++; j = *nc - 1; }
    for (; j > 0; j--) cache[j] = cache[j - 1];
    cache[0] = g;
}
/* refrel3.h:104-109: the reference base the diagonal predicts at block offset o (0..3, 4 = none) */
static int refbase(const uint8_t* ref, uint64_t ref_n, diag_t g, uint32_t o) {
    const int64_t q = g.dir ? (int64_t)g.c - (int64_t)o : (int64_t)g.c + (int64_t)o;
    if (q < 0 || (uint64_t)q >= ref_n) return 4;
    const int k = b2(g.dir ? comp_up(ref[q]) : ref[q]);
    return k < 4 ? k : 4;
}

typedef struct { uint64_t src; uint32_t dst, len, kind; } op_t;   /* RrOp (refrel_format.h:34) */

/* refrel3.h:114-169: one block's stream -> ops + literal bytes; the op count or -1 */
static int decode_block(const uint8_t* src, uint32_t n, const tab_t* T, const uint8_t* ref, uint64_t ref_n, uint32_t blen,
                        diag_t start, op_t* ops, uint32_t maxops, uint8_t* lit, uint32_t litcap) {
    static const uint8_t B[6] = {'A', 'C', 'G', 'T', 'N', 0};
    rdec d; rd_init(&d, src, n);
    if (d.bad) return -1;
    diag_t cache[4]; int nc = 1; cache[0] = start;
    int prevk = -1; uint32_t o = 0, k = 0, li = 0;
    while (o < blen) {
        const uint64_t ll = rd_val(&d, T, C_LL + kclass(prevk));
        if (d.bad || ll > blen - o) return -1;
        if (ll) {
            uint32_t p1 = 16, p2 = 16;
            for (uint32_t j = 0; j < ll; j++) {
                int c;
                if (ll <= 8) c = C_LITR + refbase(ref, ref_n, cache[0], o + j) * 2 + (j == 0 ? 1 : 0);
                else c = C_LIT2 + (p1 == 16 ? 16 : (int)(p2 == 16 ? p1 : p2 * 4 + p1) % 16);
                const uint32_t s = rd_sym(&d, T, c);
                if (li + j >= litcap) return -1;
                lit[li + j] = s < 5 ? B[s] : (uint8_t)rd_raw(&d, 8);
                p2 = p1; p1 = s < 4 ? s : 0;
            }
            if (k >= maxops) return -1;
            ops[k].kind = 0; ops[k].src = li; ops[k].dst = o; ops[k].len = (uint32_t)ll; k++;
            li += (uint32_t)ll; o += (uint32_t)ll;
        }
        if (o == blen) break;
        const int kind = (int)rd_sym(&d, T, C_KIND + llc(ll) * 4 + kclass(prevk));
        uint64_t p = 0; uint32_t dir = 0; int ki = 0; int64_t dd = 0; uint64_t dist = 0;
        if (kind == K_CONT || kind == K_DELTA) { if (kind == K_DELTA) dd = unzz(rd_val(&d, T, C_DELTA + (ll == 0 ? 0 : 1))); }
        else if (kind == K_REP) { ki = 1 + (int)rd_sym(&d, T, C_REPK); dd = unzz(rd_val(&d, T, C_REPD)); if (ki >= nc) return -1; }
        else if (kind == K_ABS) { dir = rd_sym(&d, T, C_DIR); p = rd_raw(&d, 32); }
        else if (kind == K_SELF) dist = rd_val(&d, T, C_SELF);
        else if (kind == K_FLIP) { ki = (int)rd_sym(&d, T, C_FLIPK); dd = unzz(rd_val(&d, T, C_FLIPD)); if (ki >= nc) return -1; }
        else return -1;
        const uint64_t L = rd_val(&d, T, C_LEN + kind) + MINL;
        if (d.bad || L > blen - o) return -1;
        uint32_t okind; uint64_t osrc;
        if (kind == K_SELF) { if (dist == 0 || dist > o) return -1; okind = 2; osrc = o - dist; }
        else {
            if (kind == K_FLIP) { const diag_t g = cache[ki]; dir = g.dir ^ 1; const int64_t e = dlocus(g, o) + dd; if (e < 0) return -1; p = (uint64_t)e; }
            else if (kind != K_ABS) { const diag_t g = cache[kind == K_REP ? ki : 0]; dir = g.dir; const int64_t e = dexp(g, o, L) + dd; if (e < 0) return -1; p = (uint64_t)e; }
            if (p > ref_n || L > ref_n - p) return -1;
            okind = dir ? 3 : 1; osrc = p;
            dpush(cache, &nc, dmake(dir, p, o, L));
        }
        if (k >= maxops) return -1;
        ops[k].kind = okind; ops[k].src = osrc; ops[k].dst = o; ops[k].len = (uint32_t)L; k++;
        o += (uint32_t)L; prevk = kind;
    }
    if (d.bad || d.x != RL || d.p != d.e) return -1;
    return (int)k;
}

/* pv_v1.h:65-72 (exec_ops) */
static void exec_ops(const op_t* ops, int n, const uint8_t* lit, const uint8_t* ref, uint8_t* out) {
    for (int k = 0; k < n; k++) {
        const op_t* q = &ops[k];
        if (q->kind == 0) memcpy(out + q->dst, lit + q->src, q->len);
        else if (q->kind == 1) memcpy(out + q->dst, ref + q->src, q->len);
        else if (q->kind == 2) { for (uint32_t j = 0; j < q->len; j++) out[q->dst + j] = out[q->src + j]; }
        else { const uint64_t r = q->src + q->len - 1; for (uint32_t j = 0; j < q->len; j++) out[q->dst + j] = comp_up(ref[r - j]); }
    }
}

/* ---- the reference ---- */
struct pvo_ref { uint8_t* buf; uint64_t n; uint8_t sha[32]; };

static int slurp(const char* path, uint8_t** out, uint64_t* n, char* err, size_t errlen) {
    FILE* f = fopen(path, "rb");
    if (!f) { snprintf(err, errlen, "%s: cannot open", path); return 1; }
    fseek(f, 0, SEEK_END); const long s = ftell(f); fseek(f, 0, SEEK_SET);
    uint8_t* b = (uint8_t*)malloc((size_t)s + 64);
    const size_t r = fread(b, 1, (size_t)s, f); fclose(f);
    if (r != (size_t)s) { free(b); snprintf(err, errlen, "%s: short read", path); return 1; }
    *out = b; *n = (uint64_t)s; return 0;
}

/* pv_v1.h:42-53 (fasta_bases_inplace): headers and line ends dropped, a..z upper-cased */
static int fasta_bases(uint8_t* buf, uint64_t n, const char* path, uint64_t* count, char* err, size_t errlen) {
    if (!n || buf[0] != '>') { snprintf(err, errlen, "%s: not FASTA (no header at byte 0)", path); return 1; }
    uint64_t i = 0, w = 0;
    while (i < n) {
        if (buf[i] == '>') {
            const uint8_t* e = (const uint8_t*)memchr(buf + i, '\n', n - i);
            if (!e) { snprintf(err, errlen, "%s: header without line end", path); return 1; }
            i = (uint64_t)(e - buf) + 1; continue;
        }
        const uint8_t* e = (const uint8_t*)memchr(buf + i, '\n', n - i);
        if (!e) { snprintf(err, errlen, "%s: no final line end", path); return 1; }
        const uint64_t le = (uint64_t)(e - buf);
        for (uint64_t k = i; k < le; k++) { const uint8_t c = buf[k]; buf[w++] = (c >= 'a' && c <= 'z') ? (uint8_t)(c - 32) : c; }
        i = le + 1;
    }
    *count = w; return 0;
}

int pvo_ref_load(const char* path, pvo_ref** out, char* err, size_t errlen) {
    uint8_t* b; uint64_t n;
    if (slurp(path, &b, &n, err, errlen)) return 1;
    uint64_t cnt;
    if (fasta_bases(b, n, path, &cnt, err, errlen)) { free(b); return 1; }
    pvo_ref* r = (pvo_ref*)calloc(1, sizeof *r);
    r->buf = b; r->n = cnt;
    SHA256(b, cnt, r->sha);
    *out = r; return 0;
}
void pvo_ref_free(pvo_ref* r) { if (r) { free(r->buf); free(r); } }
uint64_t pvo_ref_n(const pvo_ref* r) { return r->n; }
const uint8_t* pvo_ref_bases(const pvo_ref* r) { return r->buf; }
void pvo_ref_sha256(const pvo_ref* r, uint8_t out[32]) { memcpy(out, r->sha, 32); }

/* ---- the archive (pv_v1.h:78-146) ---- */
typedef struct { char* hdr; uint64_t len, boff; uint32_t lw; } contig_t;
struct pvo_arc {
    uint32_t Q, flags; uint64_t nbases, nb, fasta_xxh, bases_xxh, payload_bytes, file_bytes;
    contig_t* rec; uint64_t nrec;
    uint64_t* low_s; uint64_t* low_l; uint64_t nlow;
    uint64_t* hashes;
    tab_t* T; uint32_t* off; diag_t* st; uint8_t* P;
};
static uint64_t rd64(const uint8_t* p) { uint64_t v; memcpy(&v, p, 8); return v; }
static uint32_t rd32(const uint8_t* p) { uint32_t v; memcpy(&v, p, 4); return v; }

typedef struct { const uint8_t* m; size_t n, i; int bad; } meta_t;
static int need(meta_t* M, size_t k) { if (M->i + k > M->n) { M->bad = 1; return 0; } return 1; }
static uint64_t g64(meta_t* M) { if (!need(M, 8)) return 0; const uint64_t v = rd64(M->m + M->i); M->i += 8; return v; }
static uint32_t g32(meta_t* M) { if (!need(M, 4)) return 0; const uint32_t v = rd32(M->m + M->i); M->i += 4; return v; }
static uint64_t gl(meta_t* M) {
    uint64_t v = 0; int sh = 0;
    for (;;) {
        if (!need(M, 1) || sh > 63) { M->bad = 1; return 0; }
        const uint8_t c = M->m[M->i++];
        v |= (uint64_t)(c & 0x7F) << sh;
        if (!(c & 0x80)) break;
        sh += 7;
    }
    return v;
}

void pvo_arc_free(pvo_arc* X) {
    if (!X) return;
    for (uint64_t r = 0; r < X->nrec; r++) free(X->rec[r].hdr);
    free(X->rec); free(X->low_s); free(X->low_l); free(X->hashes); free(X->T); free(X->off); free(X->st); free(X->P); free(X);
}

#define REFUSE(w) do { snprintf(err, errlen, "%s: refused: %s", path, w); goto fail; } while (0)
int pvo_arc_open(const char* path, const pvo_ref* ref, pvo_arc** out, char* err, size_t errlen) {
    uint8_t* a = NULL; uint64_t n = 0; uint8_t* M = NULL;
    if (slurp(path, &a, &n, err, errlen)) return 1;
    pvo_arc* X = (pvo_arc*)calloc(1, sizeof *X);
    if (n < 136 + 2) REFUSE("short file");
    if (memcmp(a, "RFRL3V1\0", 8)) REFUSE("magic (not refrel3 v1)");
    if (rd32(a + 8) != 1) REFUSE("version");
    X->Q = rd32(a + 12);
    if (!(X->Q == 1024 || X->Q == 2048 || X->Q == 4096 || X->Q == 16384)) REFUSE("block size");
    X->flags = rd32(a + 16);
    if (X->flags & ~1u) REFUSE("unknown flags");
    if (rd32(a + 20)) REFUSE("reserved");
    X->nbases = rd64(a + 64); X->nb = rd64(a + 72); X->fasta_xxh = rd64(a + 80); X->bases_xxh = rd64(a + 88);
    const uint64_t mz = rd64(a + 96), mr = rd64(a + 104), hs = rd64(a + 112), pl = rd64(a + 120);
    const uint16_t nl = (uint16_t)(a[136] | a[137] << 8);
    const uint64_t pstart = 136ull + 2 + nl + mz + hs;
    if (mz > n || hs > n || pl > n || pstart > n || pstart + pl != n) REFUSE("section sizes");
    if (X->nb != (X->nbases + X->Q - 1) / X->Q || (X->nbases && !X->nb)) REFUSE("block count");
    if (hs != ((X->flags & 1u) ? X->nb * 8 : 0)) REFUSE("hash section size");
    {
        uint8_t* h = (uint8_t*)malloc(pstart);
        memcpy(h, a, pstart); memset(h + 128, 0, 8);
        const uint64_t hv = XXH3_64bits(h, pstart);
        free(h);
        if (hv != rd64(a + 128)) REFUSE("header XXH3");
    }
    if (memcmp(a + 24, ref->sha, 32) || rd64(a + 56) != ref->n) REFUSE("reference SHA-256 / size differs (wrong reference)");
    const uint8_t* mzp = a + 136 + 2 + nl;
    if (mr > (1ull << 32) || ZSTD_getFrameContentSize(mzp, mz) != mr) REFUSE("meta frame");
    if (ZSTD_findFrameCompressedSize(mzp, mz) != mz) REFUSE("meta frame count (exactly one zstd frame)");
    M = (uint8_t*)malloc(mr ? mr : 1);
    if (ZSTD_decompress(M, mr, mzp, mz) != mr) REFUSE("meta decompress");
    meta_t m = {M, mr, 0, 0};
    const uint32_t nr = g32(&m);
    uint64_t bo = 0;
    if (nr > mr) REFUSE("records");
    X->rec = (contig_t*)calloc(nr ? nr : 1, sizeof(contig_t));
    for (uint32_t r = 0; r < nr && !m.bad; r++) {
        const uint32_t hl = g32(&m);
        if (!need(&m, hl)) break;
        contig_t* q = &X->rec[X->nrec];
        q->hdr = (char*)malloc(hl + 1); memcpy(q->hdr, M + m.i, hl); q->hdr[hl] = 0; m.i += hl;
        q->len = g64(&m); q->lw = g32(&m);
        if (!q->lw && q->len) m.bad = 1;
        q->boff = bo; bo += q->len; X->nrec++;
    }
    if (m.bad || bo != X->nbases) REFUSE("contig table");
    const uint64_t nlw = g64(&m);
    uint64_t lst = 0;
    if (nlw > X->nbases) REFUSE("case runs");
    X->low_s = (uint64_t*)malloc((nlw ? nlw : 1) * 8); X->low_l = (uint64_t*)malloc((nlw ? nlw : 1) * 8);
    for (uint64_t k = 0; k < nlw && !m.bad; k++) {
        const uint64_t g = gl(&m), l = gl(&m);
        if (lst + g + l > X->nbases) { m.bad = 1; break; }
        X->low_s[X->nlow] = lst + g; X->low_l[X->nlow] = l; X->nlow++; lst += g + l;
    }
    if (m.bad) REFUSE("case runs");
    X->T = (tab_t*)calloc(1, sizeof(tab_t));
    for (int c = 0; c < NCTX && !m.bad; c++) {
        uint64_t sum = 0;
        for (int s = 0; s < alpha_of(c); s++) { const uint64_t f = gl(&m); if (f > MTOT) m.bad = 1; X->T->freq[c][s] = (uint16_t)f; sum += f; }
        if (sum && sum != MTOT) m.bad = 1;
    }
    if (m.bad) REFUSE("model tables");
    build_tab(X->T);
    if (pl >= (1ull << 32)) REFUSE("payload over 4 GiB (pooled offsets are 32-bit)");
    X->off = (uint32_t*)calloc(X->nb + 1, 4); X->st = (diag_t*)calloc(X->nb + 1, sizeof(diag_t));
    {
        uint64_t prevc = 0; uint32_t prevd = 0, acc = 0;
        for (uint64_t b = 0; b < X->nb && !m.bad; b++) {
            const uint64_t len = gl(&m);
            if (len > pl - acc) { m.bad = 1; break; }
            acc += (uint32_t)len; X->off[b + 1] = acc;
            const uint64_t v = gl(&m);
            const int64_t pred = b == 0 ? 0 : (int64_t)(prevd ? prevc - X->Q : prevc + X->Q);
            const uint64_t q = v >> 1;
            diag_t g; g.dir = (uint32_t)(v & 1); g.c = (uint64_t)(pred + unzz(q));
            /* the reference keeps the state packed as int64 c << 1 | dir and unpacks with an arithmetic shift
               (pv_v1.h:89,96): c keeps 63 bits, sign-extended */
            const int64_t packed = (int64_t)((uint64_t)g.c << 1) | (int64_t)(g.dir & 1);
            X->st[b].c = (uint64_t)(packed >> 1); X->st[b].dir = (uint32_t)(packed & 1);
            prevc = g.c; prevd = g.dir;
        }
        if (m.bad || m.i != mr || acc != pl) REFUSE("block table");
    }
    if (X->flags & 1u) { X->hashes = (uint64_t*)malloc((X->nb ? X->nb : 1) * 8); memcpy(X->hashes, a + 136 + 2 + nl + mz, X->nb * 8); }
    X->P = (uint8_t*)malloc(pl + 64);
    memcpy(X->P, a + pstart, pl); memset(X->P + pl, 0, 64);
    X->payload_bytes = pl; X->file_bytes = n;
    free(M); free(a);
    *out = X; return 0;
fail:
    free(M); free(a); pvo_arc_free(X);
    return 1;
}
#undef REFUSE

uint32_t pvo_arc_q(const pvo_arc* a) { return a->Q; }
uint64_t pvo_arc_nbases(const pvo_arc* a) { return a->nbases; }
uint64_t pvo_arc_nblocks(const pvo_arc* a) { return a->nb; }
uint64_t pvo_arc_payload_bytes(const pvo_arc* a) { return a->payload_bytes; }
uint64_t pvo_arc_block_payload(const pvo_arc* a, uint64_t b) { return b < a->nb ? (uint64_t)(a->off[b + 1] - a->off[b]) : 0; }
uint32_t pvo_arc_freq(const pvo_arc* a, int c, int s) { return (c >= 0 && c < NCTX && s >= 0 && s < AB) ? a->T->freq[c][s] : 0; }
int pvo_arc_block_state(const pvo_arc* a, uint64_t b, uint64_t* c, uint32_t* dir) {
    if (b >= a->nb) return 1;
    *c = a->st[b].c; *dir = a->st[b].dir;
    return 0;
}
uint64_t pvo_arc_fasta_xxh3(const pvo_arc* a) { return a->fasta_xxh; }
uint64_t pvo_arc_ncontigs(const pvo_arc* a) { return a->nrec; }
uint64_t pvo_arc_nlow(const pvo_arc* a) { return a->nlow; }
int pvo_arc_contig(const pvo_arc* a, uint64_t i, char* hdr, size_t cap, uint64_t* len, uint64_t* boff, uint32_t* lw) {
    if (i >= a->nrec) return 1;
    if (hdr && cap) { strncpy(hdr, a->rec[i].hdr, cap - 1); hdr[cap - 1] = 0; }
    *len = a->rec[i].len; *boff = a->rec[i].boff; *lw = a->rec[i].lw;
    return 0;
}

/* ---- block, window, batch (pv_v1.h:148-174, pv_core.cpp:116-136) ---- */
typedef struct { op_t* ops; uint8_t* lit; uint8_t* blk; } scratch_t;
static void scratch_init(scratch_t* S, uint32_t Q) { S->ops = (op_t*)malloc(MAXOPS * sizeof(op_t)); S->lit = (uint8_t*)malloc(Q); S->blk = (uint8_t*)malloc(Q); }
static void scratch_free(scratch_t* S) { free(S->ops); free(S->lit); free(S->blk); }

static int block_into(const pvo_arc* X, const pvo_ref* R, uint64_t b, uint8_t* out, scratch_t* S, int verify) {
    const uint32_t blen = (uint32_t)((X->nbases - b * X->Q) < X->Q ? (X->nbases - b * X->Q) : X->Q);
    const int k = decode_block(X->P + X->off[b], X->off[b + 1] - X->off[b], X->T, R->buf, R->n, blen, X->st[b], S->ops, MAXOPS,
                               S->lit, X->Q);
    if (k < 0) return 1;
    exec_ops(S->ops, k, S->lit, R->buf, out);
    if (verify && X->hashes && XXH3_64bits(out, blen) != X->hashes[b]) return 2;
    return 0;
}
int pvo_block(const pvo_arc* a, const pvo_ref* ref, uint64_t b, uint8_t* out, int verify) {
    if (b >= a->nb) return 1;
    scratch_t S; scratch_init(&S, a->Q);
    const int e = block_into(a, ref, b, out, &S, verify);
    scratch_free(&S);
    return e;
}
static size_t first_run(const pvo_arc* X, uint64_t x) {
    size_t lo = 0, hi = X->nlow;
    while (lo < hi) { const size_t m = (lo + hi) / 2; if (X->low_s[m] + X->low_l[m] <= x) lo = m + 1; else hi = m; }
    return lo;
}
static int window_with(const pvo_arc* X, const pvo_ref* R, uint64_t s, uint64_t W, int rc, int tokens, int apply_case,
                       int verify, uint8_t* out, scratch_t* S) {
    if (s + W > X->nbases || s + W < s) return 8;
    if (W) {
        for (uint64_t b = s / X->Q; b <= (s + W - 1) / X->Q; b++) {
            const int e = block_into(X, R, b, S->blk, S, verify);
            if (e) return e;
            const uint64_t bs = b * X->Q, x0 = s > bs ? s : bs, x1 = (s + W) < (bs + X->Q) ? (s + W) : (bs + X->Q);
            memcpy(out + (x0 - s), S->blk + (x0 - bs), x1 - x0);
        }
        if (apply_case && !tokens)
            for (size_t r = first_run(X, s); r < X->nlow && X->low_s[r] < s + W; r++) {
                const uint64_t x0 = s > X->low_s[r] ? s : X->low_s[r];
                const uint64_t e = X->low_s[r] + X->low_l[r], x1 = (s + W) < e ? (s + W) : e;
                for (uint64_t x = x0; x < x1; x++) out[x - s] |= 0x20;
            }
    }
    if (rc) {
        for (int64_t i = 0, j = (int64_t)W - 1; i < j; i++, j--) { const uint8_t t = comp_case(out[i]); out[i] = comp_case(out[j]); out[j] = t; }
        if (W & 1) out[W / 2] = comp_case(out[W / 2]);
    }
    if (tokens) for (uint64_t i = 0; i < W; i++) out[i] = token(out[i]);
    return 0;
}
int pvo_window(const pvo_arc* a, const pvo_ref* ref, uint64_t s, uint64_t W, int rc, int tokens, int apply_case, int verify,
               uint8_t* out) {
    scratch_t S; scratch_init(&S, a->Q);
    const int e = window_with(a, ref, s, W, rc, tokens, apply_case, verify, out, &S);
    scratch_free(&S);
    return e;
}

typedef struct {
    pvo_arc* const* arcs; int64_t narcs; const pvo_ref* ref; int64_t n; const int64_t* asm_idx; const int64_t* start;
    uint64_t W; const uint8_t* rc; int tokens, apply_case, verify; uint8_t* out; uint64_t chunk, nchunks;
    atomic_ullong next; atomic_int err;
} batch_t;
static void* batch_worker(void* arg) {
    batch_t* B = (batch_t*)arg;
    uint32_t Q = B->narcs ? B->arcs[0]->Q : 1024;
    for (int64_t i = 1; i < B->narcs; i++) if (B->arcs[i]->Q > Q) Q = B->arcs[i]->Q;
    scratch_t S; scratch_init(&S, Q);
    for (;;) {
        const uint64_t c = atomic_fetch_add(&B->next, 1);
        if (c >= B->nchunks || atomic_load(&B->err)) break;
        const uint64_t w1 = (c + 1) * B->chunk < (uint64_t)B->n ? (c + 1) * B->chunk : (uint64_t)B->n;
        for (uint64_t w = c * B->chunk; w < w1; w++) {
            const int64_t ai = B->asm_idx[w];
            int e = (ai < 0 || ai >= B->narcs || B->start[w] < 0) ? 8
                  : window_with(B->arcs[ai], B->ref, (uint64_t)B->start[w], B->W, B->rc ? B->rc[w] : 0, B->tokens, B->apply_case,
                                B->verify, B->out + w * B->W, &S);
            if (e) { int z = 0; atomic_compare_exchange_strong(&B->err, &z, e); break; }
        }
    }
    scratch_free(&S);
    return NULL;
}
int pvo_windows(pvo_arc* const* arcs, int64_t narcs, const pvo_ref* ref, int64_t n, const int64_t* asm_idx, const int64_t* start,
                uint64_t W, const uint8_t* rc, int tokens, int apply_case, int verify, int threads, uint8_t* out) {
    if (n <= 0) return 0;
    if (threads < 1) threads = 1;
    batch_t B; memset(&B, 0, sizeof B);
    B.arcs = arcs; B.narcs = narcs; B.ref = ref; B.n = n; B.asm_idx = asm_idx; B.start = start; B.W = W; B.rc = rc;
    B.tokens = tokens; B.apply_case = apply_case; B.verify = verify; B.out = out;
    B.chunk = ((uint64_t)n + (uint64_t)threads * 4 - 1) / ((uint64_t)threads * 4);
    if (!B.chunk) B.chunk = 1;
    B.nchunks = ((uint64_t)n + B.chunk - 1) / B.chunk;
    atomic_init(&B.next, 0); atomic_init(&B.err, 0);
    if ((uint64_t)threads > B.nchunks) threads = (int)B.nchunks;
    pthread_t* th = (pthread_t*)malloc(sizeof(pthread_t) * (size_t)threads);
    for (int t = 0; t < threads; t++) pthread_create(&th[t], NULL, batch_worker, &B);
    for (int t = 0; t < threads; t++) pthread_join(th[t], NULL);
    free(th);
    return atomic_load(&B.err);
}

/* ---- full decode -> FASTA (pv_core.cpp:138-159) and the FASTA hash of a base stream (pv_core.cpp:167-176) ---- */
static uint64_t fasta_size(const pvo_arc* X) {
    uint64_t size = 0;
    for (uint64_t r = 0; r < X->nrec; r++) {
        const contig_t* c = &X->rec[r];
        size += 2 + strlen(c->hdr) + c->len + (c->lw ? (c->len + c->lw - 1) / c->lw : 0);
    }
    return size;
}
int pvo_fasta(const pvo_arc* X, const pvo_ref* R, int verify, uint8_t* out, uint64_t cap, uint64_t* size) {
    const uint64_t sz = fasta_size(X);
    *size = sz;
    if (!out) return 0;
    if (cap < sz) return 4;
    uint8_t* B = (uint8_t*)malloc(X->nbases + 64);
    scratch_t S; scratch_init(&S, X->Q);
    int err = 0;
    for (uint64_t b = 0; b < X->nb && !err; b++) err = block_into(X, R, b, B + b * X->Q, &S, verify);
    scratch_free(&S);
    if (!err) {
        for (uint64_t r = 0; r < X->nlow; r++) for (uint64_t x = X->low_s[r]; x < X->low_s[r] + X->low_l[r]; x++) B[x] |= 0x20;
        uint8_t* p = out;
        for (uint64_t r = 0; r < X->nrec; r++) {
            const contig_t* c = &X->rec[r];
            const size_t hl = strlen(c->hdr);
            *p++ = '>'; memcpy(p, c->hdr, hl); p += hl; *p++ = '\n';
            for (uint64_t x = 0; x < c->len; x += c->lw) {
                const uint64_t k = c->lw < c->len - x ? c->lw : c->len - x;
                memcpy(p, B + c->boff + x, k); p += k; *p++ = '\n';
            }
        }
        if ((uint64_t)(p - out) != sz) err = 4;
        else if (verify && XXH3_64bits(out, sz) != X->fasta_xxh) err = 3;
    }
    free(B);
    return err;
}
uint64_t pvo_fasta_xxh3(const pvo_arc* X, const uint8_t* bases) {
    XXH3_state_t* h = XXH3_createState();
    XXH3_64bits_reset(h);
    for (uint64_t r = 0; r < X->nrec; r++) {
        const contig_t* c = &X->rec[r];
        const uint8_t gt = '>', nl = '\n';
        XXH3_64bits_update(h, &gt, 1); XXH3_64bits_update(h, c->hdr, strlen(c->hdr)); XXH3_64bits_update(h, &nl, 1);
        for (uint64_t x = 0; x < c->len; x += c->lw) {
            const uint64_t k = c->lw < c->len - x ? c->lw : c->len - x;
            XXH3_64bits_update(h, bases + c->boff + x, k); XXH3_64bits_update(h, &nl, 1);
        }
    }
    const uint64_t v = XXH3_64bits_digest(h);
    XXH3_freeState(h);
    return v;
}
