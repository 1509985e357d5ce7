/* pv_oracle.h - TEST INFRASTRUCTURE ONLY. A CPU restatement of the reference's refrel3 v1 reader and decoder
 * (panvram 1.0.1: csrc/refrel3.h, refrel_format.h, pv_v1.h and pv_core.cpp), used as the parity checker
 * of the CUDA path. Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may load it; the product
 * (panvram_b200) never links, imports or calls it.
 *
 * Pinned against the reference's own fixtures (the tests/data archives with the header's source-FASTA XXH3, and windows
 * produced by the reference's compiled CPU decoder, committed under tests/golden/). */
#pragma once
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct pvo_ref pvo_ref;
typedef struct pvo_arc pvo_arc;

/* reference FASTA -> upper-case base stream + SHA-256 (pv_core.cpp:35-41, pv_v1.h:42-53) */
int pvo_ref_load(const char* path, pvo_ref** out, char* err, size_t errlen);
void pvo_ref_free(pvo_ref* r);
uint64_t pvo_ref_n(const pvo_ref* r);
const uint8_t* pvo_ref_bases(const pvo_ref* r);
void pvo_ref_sha256(const pvo_ref* r, uint8_t out[32]);

/* archive open with every FORMAT section-5 check (pv_v1.h:99-146); err gets "<path>: refused: <why>" */
int pvo_arc_open(const char* path, const pvo_ref* ref, pvo_arc** out, char* err, size_t errlen);
void pvo_arc_free(pvo_arc* a);
uint32_t pvo_arc_q(const pvo_arc* a);
uint64_t pvo_arc_nbases(const pvo_arc* a);
uint64_t pvo_arc_nblocks(const pvo_arc* a);
uint64_t pvo_arc_payload_bytes(const pvo_arc* a);
uint64_t pvo_arc_block_payload(const pvo_arc* a, uint64_t b);   /* payload bytes of block b */
int pvo_arc_block_state(const pvo_arc* a, uint64_t b, uint64_t* c, uint32_t* dir);   /* start diagonal of block b */
uint32_t pvo_arc_freq(const pvo_arc* a, int c, int s);        /* model frequency of symbol s in context c */
uint64_t pvo_arc_fasta_xxh3(const pvo_arc* a);
uint64_t pvo_arc_ncontigs(const pvo_arc* a);
/* contig i: header copied into hdr (NUL-terminated, truncated to cap), length, base offset, line width */
int pvo_arc_contig(const pvo_arc* a, uint64_t i, char* hdr, size_t cap, uint64_t* len, uint64_t* boff, uint32_t* lw);
uint64_t pvo_arc_nlow(const pvo_arc* a);

/* block b, upper case, into out (Q bytes of room): 0 ok, 1 decode error, 2 block XXH3 mismatch (verify)
 * (pv_v1.h:150-158) */
int pvo_block(const pvo_arc* a, const pvo_ref* ref, uint64_t b, uint8_t* out, int verify);
/* bases [s, s+W) with case runs (unless tokens), then reverse complement, then tokens (pv_v1.h:164-174,
 * pv_core.cpp:129-132): 0 ok, 1 decode error, 2 block hash, 8 window outside the assembly */
int pvo_window(const pvo_arc* a, const pvo_ref* ref, uint64_t s, uint64_t W, int rc, int tokens, int apply_case,
               int verify, uint8_t* out);
/* a batch over many archives on `threads` host threads (pv_core.cpp:116-136): out is n*W bytes; rc may be NULL;
 * returns the first non-zero window code */
int pvo_windows(pvo_arc* const* arcs, int64_t narcs, const pvo_ref* ref, int64_t n, const int64_t* asm_idx,
                const int64_t* start, uint64_t W, const uint8_t* rc, int tokens, int apply_case, int verify, int threads,
                uint8_t* out);
/* full decode -> FASTA bytes (pv_core.cpp:138-159); size query with out == NULL. 0 ok, 1 decode, 2 block hash,
 * 3 FASTA XXH3 differs from the header, 4 size */
int pvo_fasta(const pvo_arc* a, const pvo_ref* ref, int verify, uint8_t* out, uint64_t cap, uint64_t* size);
/* XXH3 of the FASTA rebuilt from a decoded base stream with case applied (pv_core.cpp:167-176) */
uint64_t pvo_fasta_xxh3(const pvo_arc* a, const uint8_t* bases);

#ifdef __cplusplus
}
#endif
