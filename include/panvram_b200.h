/* panvram_b200.h - the C ABI of panvram_b200: a B200-native decoder for panvram's refrel3 v1 random-access window
 * path. Plain pointers and sizes; no torch types. Every entry point names the reference interface it replaces
 * (panvram 1.0.1, paths inside that project). Device pointers are CUDA device addresses on the current device.
 *
 * Error convention: functions return PV_OK (0) or a PV_E* code; pv_last_error() gives the message of the calling
 * thread's last failure. Format refusals carry the reference's text ("<path>: refused: <why>", pv_v1.h:101). */
#pragma once
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define PV_OK 0
#define PV_EFORMAT 1      /* archive / reference refused (the reference's FormatError, pv_core.cpp:196) */
#define PV_EARG 2         /* argument error (the reference's TORCH_CHECK -> RuntimeError, pv_cuda.cu:119-128) */
#define PV_ECUDA 3        /* a CUDA runtime call failed */
#define PV_EIO 4          /* file read error */

/* status bits a window call ORs into its int32 status word (pv_cuda.cu:37) */
#define PV_STATUS_DECODE 1    /* a touched block failed to decode (corrupt archive) */
#define PV_STATUS_WAIT 4      /* a bounded wait inside a kernel expired */
#define PV_STATUS_WINDOW 8    /* a window lies outside its assembly (or names no assembly) */

#define PV_NCTX 61                 /* refrel3 model contexts (refrel3.h:24) */
#define PV_TAB_MAX_BYTES 8208      /* largest per-assembly device decode table (layout: panvram_b200/csrc/pv_layout.h) */

/* Per assembly, device record (64 bytes). */
typedef struct pv_asm_rec {
    uint64_t nbases;      /* bases of the assembly's stream (header offset 64) */
    uint64_t blk_base;    /* its first entry in pv_dev_cohort.blocks */
    uint64_t nb;          /* blocks = ceil(nbases / Q) */
    uint64_t low_base;    /* its first lower-case run in pv_dev_cohort.low */
    uint64_t low_cnt;     /* its lower-case run count */
    uint64_t tab_off;     /* its decode table: byte offset in pv_dev_cohort.tabs (16-byte aligned) */
    uint64_t tab_bytes;   /* and size (a multiple of 16) */
    uint64_t grp_base;    /* compact block table: its first group in pv_dev_cohort.groups */
} pv_asm_rec;

/* Opt-in compact resident forms (pv_core_open's packed_reference / compact_blocks; the reference's PackedRef and
 * CompactTab, pv_compact.h:1-48): same archives, same output, less device memory. */

/* packed reference: 2 bits per base (A 0, C 1, G 2, T 3; 16 bases per 32-bit word, base q at bits 2 (q mod 16) of word
 * q / 16) plus the runs of any other byte (N, IUPAC codes), sorted and disjoint; a run is one byte repeated. The run
 * array ends with a sentinel run starting at UINT64_MAX (not counted in pnruns). */
typedef struct pv_ref_run {
    uint64_t start;
    uint32_t len;
    uint32_t byte;
} pv_ref_run;
#define PV_REF_BUCKET_SHIFT 12     /* pv_dev_cohort.pidx[k]: the first run ending after position k << 12 */

/* compact block table: per group of PV_BLK_GROUP consecutive blocks of one assembly a 32-byte record, per block 32
 * bits: payload length (16 bits) | state code << 16. The state code of a block after the first of its group is its
 * start diagonal's difference from the chain prediction (previous block's c + Q forward, - Q reverse) times 2 plus its
 * strand, or PV_CODE_EXC: then the state is exception entry exc_base + (exceptions before it in the group). */
#define PV_BLK_GROUP 32
#define PV_CODE_EXC (-32768)
typedef struct pv_blk_group {
    uint64_t off;          /* payload offset of the group's first block in pv_dev_cohort.payload */
    int64_t state;         /* its start state c << 1 | dir */
    uint32_t exc_mask;     /* blocks of the group whose state is an exception entry */
    uint32_t exc_base;     /* the first of them in pv_dev_cohort.bexc */
    uint32_t cache_mask;   /* blocks of the group served from pv_dev_cohort.cache */
    uint32_t cache_base;   /* cache slot of the first of them; the next ones follow in block order */
} pv_blk_group;

/* Decoder checkpoint (32 bytes): the refrel3 decoder's whole state at an event boundary inside a block (the top of the
 * event loop of refrel3.h:119-159), so that a decode can start there instead of at the block's start. The checkpoint
 * index of a cohort holds, per block, Q / S of them (S = 1 << pv_dev_cohort.ckpt_shift, the stride): checkpoint j is
 * the state at the last event boundary at or before block offset j S (checkpoint 0 is the block's start). Built on
 * the device at open by pv_index_build, which decodes every block once and so also validates it: a block that fails
 * to decode has PV_CKPT_BAD in all its checkpoints, and a window touching it reports PV_STATUS_DECODE as the
 * reference's decode of that block would. The diagonal cache entries are stored as c + PV_CKPT_BIAS in 39 bits. */
typedef struct pv_ckpt {
    uint32_t xs;          /* rANS state (24 bits) | previous kind + 1 << 24 (3 bits) | diagonal count - 1 << 27 (2 bits) */
    uint32_t p;           /* bits 0..31 of the position in the pooled payload of the next stream byte to read (or, with
                           * PV_CKPT_CACHED, the block's row in pv_dev_cohort.cache) */
    uint32_t clo[4];      /* diagonal k (most recent first): bits 0..31 of c + PV_CKPT_BIAS */
    uint8_t chi[4];       /* bits 32..38 of c + PV_CKPT_BIAS | strand << 7 */
    uint16_t o;           /* block offset of the event boundary */
    uint16_t flags;       /* PV_CKPT_BAD, PV_CKPT_CACHED | bits 32..39 of the payload position << 8 */
} pv_ckpt;
#define PV_CKPT_BIAS (1ll << 20)
#define PV_CKPT_BAD 1u        /* the block failed to decode */
#define PV_CKPT_CACHED 2u     /* the block is served from the block cache (no decoder state) */

/* The pooled cohort as the window kernel reads it (device addresses). Built on the host by pv_core_pools() and
 * uploaded by the caller; it replaces the reference's pooled tensors P, pay_base, off, st, tab, blk_base, nbases,
 * low_s, low_l, low_base, low_cnt, ref (pv_core.cpp:65-90) that windows_cuda takes (pv_cuda.cu:153-162). */
typedef struct pv_dev_cohort {
    const uint8_t* ref;          /* decoded reference, first base; 64 zero bytes readable on each side */
    uint64_t ref_n;
    const uint8_t* payload;      /* pooled rANS streams; 64 zero bytes readable after the end */
    const uint64_t* blocks;      /* 2 words per block: payload offset | payload length << 40, start state c << 1 | dir */
    const pv_asm_rec* asms;      /* [nasm] */
    const uint8_t* tabs;         /* pooled decode tables (pv_asm_rec.tab_off / tab_bytes) */
    uint64_t tab_max;            /* the largest table's bytes */
    const uint64_t* low;         /* pooled lower-case runs, [start, end) pairs, sorted per assembly */
    const uint8_t* cache;        /* decoded blocks (Q bytes each, upper case), 64 readable bytes on each side, or NULL */
    int64_t nasm;
    uint32_t Q;                  /* block size of the cohort: 1024, 2048, 4096 or 16384 */
    uint32_t pad;
    /* packed reference (packed != 0; ref is then NULL) */
    const uint32_t* pref;        /* ceil(ref_n / 16) words + 4 zero words */
    const pv_ref_run* pruns;     /* [pnruns] */
    const uint32_t* pidx;        /* [(ref_n >> PV_REF_BUCKET_SHIFT) + 2] */
    uint64_t pnruns;
    /* compact block table (compact != 0; blocks is then NULL) */
    const pv_blk_group* groups;
    const uint32_t* btab;        /* per pooled block: length | code << 16 */
    const int64_t* bexc;         /* exception states, in block order */
    uint32_t packed, compact;
    /* checkpoint index (pv_index_build), or NULL: then every window item decodes its block from the block's start to
     * its end, validating it as it goes */
    const pv_ckpt* ckpt;         /* [pooled blocks << (log2 Q - ckpt_shift)] */
    uint32_t ckpt_shift;         /* log2 of the stride S (8 <= ckpt_shift <= log2 Q) */
    uint32_t pad2;
    /* per pooled block, its assembly's first lower-case run (index from the assembly's low_base) that ends after the
     * block's start (pv_index_build), or NULL: then the window kernels binary-search the runs */
    const uint32_t* brun;
    /* the reference reverse-complemented (pv_rc_reference: rcref[i] = complement of ref[ref_n - 1 - i]), 64 readable
     * bytes on each side, or NULL: with it a reverse-complement copy is read forward from it (byte form only) */
    const uint8_t* rcref;
} pv_dev_cohort;

/* Block table word 0 of a block served from pv_dev_cohort.cache: cache slot | PV_BLOCK_CACHED << 40 (the payload
 * length field 0xFFFFFE never occurs for a block stream; 0xFFFFFF marks a stream too long to be valid). */
#define PV_BLOCK_CACHED 0xFFFFFEull

/* The host-side pooled arrays (pv_core_pools); byte sizes give the device allocation for each. The device `ref`
 * pointer is (device copy of ref_padded) + 64. */
typedef struct pv_host_pools {
    const uint8_t* ref_padded; uint64_t ref_padded_bytes;
    const uint8_t* payload; uint64_t payload_bytes;
    const uint64_t* blocks; uint64_t blocks_bytes;
    const pv_asm_rec* asms; uint64_t asms_bytes;
    const uint8_t* tabs; uint64_t tabs_bytes; uint64_t tab_max;
    const uint64_t* low; uint64_t low_bytes;
    const int64_t* ctg_asm; const int64_t* ctg_local; const int64_t* ctg_boff; const int64_t* ctg_len; uint64_t ncontigs;
    /* the compact forms, when opened with them (then ref_padded / blocks are NULL with 0 bytes) */
    const uint32_t* pref; uint64_t pref_bytes;
    const pv_ref_run* pruns; uint64_t pruns_bytes; uint64_t pnruns;
    const uint32_t* pidx; uint64_t pidx_bytes;
    const pv_blk_group* groups; uint64_t groups_bytes;
    const uint32_t* btab; uint64_t btab_bytes;
    const int64_t* bexc; uint64_t bexc_bytes;
    uint32_t packed, compact;
} pv_host_pools;

typedef struct pv_asm_info {
    uint32_t Q; uint32_t block_hashes;
    uint64_t bases, blocks, file_bytes, payload_bytes, contigs, lower_case_runs;
    uint64_t fasta_xxh3, bases_xxh3;
} pv_asm_info;

typedef struct pv_core pv_core;

const char* pv_last_error(void);

/* ---- host: open, pool, describe (replaces panvram._C.Core, pv_core.cpp:23-183, 195-212) ---- */

/* Core(reference, paths, threads, packed_reference, compact_blocks) (pv_core.cpp:32-50, bound at :198-199): read the
 * reference FASTA (upper-cased, SHA-256), open every archive with all FORMAT section-5 checks (pv_v1.h:99-146),
 * one block size per cohort, pool the arrays into the device layout. threads 0 = all host threads.
 * packed_reference: keep the reference as pv_ref_run runs + 2-bit words (pv_compact.h:19-28); compact_blocks: keep the
 * block table as pv_blk_group records + 32 bits per block (pv_compact.h:30-46; a block payload over 65535 B is
 * refused, pv_core.cpp:102). Windows are the same in every form. */
int pv_core_open(const char* reference, const char* const* paths, int64_t npaths, int threads, int packed_reference,
                 int compact_blocks, pv_core** out);
void pv_core_free(pv_core* c);
int64_t pv_core_n(const pv_core* c);                    /* Core.n (pv_core.cpp:208) */
uint32_t pv_core_q(const pv_core* c);                   /* Core.Q (:205) */
uint64_t pv_core_ref_bases(const pv_core* c);           /* Core.ref_bases (:209) */
void pv_core_ref_sha256(const pv_core* c, char hex[65]); /* Core.ref_sha256 (:210) */
int pv_core_pools(const pv_core* c, pv_host_pools* out);/* Core.pools (pv_core.cpp:177-182) */
/* Free the host copies of the reference and of the pooled payload (plain and packed forms), once the caller has
 * copied them to its device: they are read for nothing else. pv_core_pools then reports them empty (earlier views of
 * them dangle); the rest of the core - block table, lower-case runs, contigs, decode tables, every archive's
 * metadata - stays. No counterpart in the reference, whose Core keeps them. */
void pv_core_release_uploaded(pv_core* c);
int pv_core_info(const pv_core* c, int64_t asm_index, pv_asm_info* out);   /* Core.info (pv_core.cpp:161-163) */
/* reference name and path strings of Core.info; NUL-terminated, truncated to cap */
int pv_core_info_strings(const pv_core* c, int64_t asm_index, char* path, size_t path_cap, char* refname, size_t ref_cap);
/* Core.contigs (pv_core.cpp:160): contig i of assembly a -> header, name, length, base offset, line width */
int64_t pv_core_ncontigs(const pv_core* c, int64_t asm_index);
int pv_core_contig(const pv_core* c, int64_t asm_index, int64_t i, char* hdr, size_t hdr_cap, char* name, size_t name_cap,
                   uint64_t* len, uint64_t* boff, uint32_t* line_width);
/* Core.fasta_xxh3 (pv_core.cpp:167-176): XXH3 of the FASTA rebuilt from a decoded base stream (case applied) */
int pv_core_fasta_xxh3(const pv_core* c, int64_t asm_index, const uint8_t* bases, uint64_t nbases, uint64_t* out_hash);
/* FASTA bytes rebuilt from a decoded base stream (case applied): size query with out == NULL; the rebuild half of
 * Core.fasta (pv_core.cpp:138-159), whose decode half runs on the GPU here */
int pv_core_fasta_write(const pv_core* c, int64_t asm_index, const uint8_t* bases, uint64_t nbases, uint8_t* out,
                        uint64_t cap, uint64_t* size);
/* block XXH3 check of a decoded upper-case stream (flag bit 0 archives; pv_v1.h:156): first bad block or -1 */
int pv_core_check_block_hashes(const pv_core* c, int64_t asm_index, const uint8_t* upper_bases, uint64_t nbases,
                               int64_t* first_bad);
/* lower-case runs of assembly a applied in place to a decoded upper-case stream (pv_core.cpp:149) */
int pv_core_apply_case(const pv_core* c, int64_t asm_index, uint8_t* bases, uint64_t nbases);
/* sha256_file_bases (pv_core.cpp:211): SHA-256 of a FASTA's upper-cased base stream, as hex */
int pv_sha256_file_bases(const char* path, char hex[65]);

/* ---- device: the window decode (replaces windows_cuda / windows_cuda2, pv_cuda.cu:117-179) ---- */

/* out[i, 0:W] = bases [start[i], start[i] + W) of assembly asm[i], lower-case runs applied (apply_case, skipped when
 * tokens), reverse-complemented where rc[i] != 0 (rc may be NULL), then mapped to tokens A/a 0 C/c 1 G/g 2 T/t 3
 * else 4 when tokens. asm, start: int64 [n] device; out: uint8 [n * W] device; status: int32 device word that the
 * call ORs PV_STATUS_* bits into (the caller zeroes it); work: device scratch of at least pv_windows_work_bytes()
 * bytes, 16-byte aligned (the split form's work queue, plan of decoded items and general-path list, and block
 * buffers; nothing in it needs to start at zero; calls running at the same time need their own). Launches on `stream` (a cudaStream_t), asynchronous. Same argument checks as pv_cuda.cu:119-128:
 * W in [0, 2^31), n >= 0. */
int pv_windows(const pv_dev_cohort* cohort, const int64_t* asm_index, const int64_t* start, int64_t n, int64_t W,
               const uint8_t* rc, int tokens, int apply_case, uint8_t* out, int32_t* status, void* work, size_t work_bytes,
               void* stream);
/* device scratch one pv_windows / pv_windows_ex call with these sizes needs (0 for an empty call) */
size_t pv_windows_work_bytes(const pv_dev_cohort* cohort, int64_t n, int64_t W);

/* pv_windows with flags and an optional per-window status. PV_WIN_BLOCK_PATH routes every block through the general
 * path (the whole block materialised in shared memory, ops executed in order) instead of only the blocks that need
 * it; the output is the same, it is for testing that path on every input. wstatus (NULL or uint8 [n], zeroed by the
 * caller) receives the PV_STATUS_* bits of each window; the cohort's block cache is filled this way at open. */
#define PV_WIN_BLOCK_PATH 1u
/* The kernels a call runs: by default the one-kernel form (one warp per item decodes on one lane and emits) while the
 * call has fewer than 4,608 work items (3,072 when the item cell is 16,384 bases; items = n x (ceil(W / cell) + 1), the
 * cell being the checkpoint stride of a cohort with an index, else its block size), else three launches
 * (pv_decode_kernel: one item per lane, as many per warp as keep about 3,072 decode warps busy, at most 32;
 * pv_emit_kernel: persistent, each warp taking the next decoded item from a queue and writing it; pv_heavy_kernel: the
 * items that need the general path, usually none). PV_WIN_FUSED / PV_WIN_SPLIT force one form; the output is the
 * same. */
#define PV_WIN_FUSED 2u
#define PV_WIN_SPLIT 4u
/* For testing the expired-wait path (status 4) without a fault: every kernel's bounded wait on its shared-memory bulk
 * copies is made to expire - its barrier expects 16 bytes that no copy brings, and the wait's bound is short - so each
 * item that stages copies reports PV_STATUS_WAIT and writes nothing; the kernel then completes the missing 16 bytes with
 * one more copy and waits until every copy has landed before it returns. The context stays usable. Only the one-kernel
 * form (pv_windows_kernel) stages copies; the split form's kernels wait on none, and there the flag changes nothing. */
#define PV_WIN_TEST_WAIT 16u
/* the split form's decode warps: PV_WIN_DEC_LANES(k) runs k items per warp (one per lane, k in 1..32) instead of
 * the size rule's choice; the output is the same */
#define PV_WIN_DEC_LANES_SHIFT 8
#define PV_WIN_DEC_LANES(k) ((uint32_t)(k) << PV_WIN_DEC_LANES_SHIFT)
int pv_windows_ex(const pv_dev_cohort* cohort, const int64_t* asm_index, const int64_t* start, int64_t n, int64_t W,
                  const uint8_t* rc, int tokens, int apply_case, uint32_t flags, uint8_t* out, int32_t* status, uint8_t* wstatus,
                  void* work, size_t work_bytes, void* stream);

/* pv_windows with the token map fused into the store. The reference maps tokens to a model's ids in a second pass
 * over the decoded tokens (tools/megatron/panvram_loader.py:97, `lut5[raw.long()]`, after windows(tokens=True)); here
 * out[i, 0:W] = ids[token] as int64, token as pv_windows computes it (A/a 0, C/c 1, G/g 2, T/t 3, else 4; of the
 * complement where rc[i] != 0), written once. out: int64 [n * W] device, 16-byte aligned; ids: 5 values (host). */
int pv_windows_ids(const pv_dev_cohort* cohort, const int64_t* asm_index, const int64_t* start, int64_t n, int64_t W,
                   const uint8_t* rc, const int64_t* ids, int64_t* out, int32_t* status, void* work, size_t work_bytes,
                   void* stream);

/* Work items of a pv_windows call with these sizes: (window, cell) pairs, the cell being the cohort's checkpoint stride
 * (or its block without an index); n x (ceil(W / cell) + 1), some of them empty. */
size_t pv_windows_items(const pv_dev_cohort* cohort, int64_t n, int64_t W);
/* pv_windows_ex without a per-window status, and with a per-item trace (no counterpart in the reference, which has
 * none; its logs time the decode ad hoc with clock64 / %globaltimer): trace (device uint64 [trace_records x 8],
 * trace_records >= pv_windows_items, zeroed by the caller) receives for item i the %globaltimer time (ns) at which it
 * reached each phase - word 0 start, 1 located (block, checkpoint, lower-case runs), 2 its decode starts (fused
 * kernel: after its staged copies landed), 3 decoded, 4 taken by the emission kernel (split form), 5 its header in
 * the emission warp's slot, 6 its bytes written - and in word 7: SM | item state << 8 | form << 12 (1 fused, 2 split) | decode
 * from a checkpoint << 14 | ops << 16 | literal bytes << 32 | bases decoded << 48. A phase the item did not reach
 * stays 0. Same output as pv_windows_ex; the timer reads add a little time. */
int pv_windows_trace(const pv_dev_cohort* cohort, const int64_t* asm_index, const int64_t* start, int64_t n, int64_t W,
                     const uint8_t* rc, int tokens, int apply_case, uint32_t flags, uint8_t* out, int32_t* status, void* work,
                     size_t work_bytes, uint64_t* trace, size_t trace_records, void* stream);

/* The coordinate arithmetic of Cohort.sample between its draws and its pv_windows call (panvram/cohort.py:177-189 and 193-194,
 * there six torch ops), as one launch. For window i: contig k = the first index with cum[k] > u[i] (searchsorted
 * right; u[i] in [0, cum[nctg-1]), cum the inclusive prefix sum of valid[], valid[k] = max(0, contig length - W + 1)),
 * pos = u[i] - (cum[k] - valid[k]); asm_index[i] = ctg_asm[k], start[i] = ctg_boff[k] + pos. rc_mode 0: no strand
 * (rc untouched, may be NULL), 1: rc[i] = 1, 2: rc[i] = (r[i] < p) for the sample's rand() draw r. coords (NULL or int64
 * [n, 4]): (assembly, ctg_local[k], pos, strand). status (NULL or an int32 device word) is set to 0 first, so the
 * pv_windows call that follows on the stream can OR into it. All pointers device; asynchronous on `stream`. */
int pv_sample_coords(const int64_t* cum, const int64_t* valid, const int64_t* ctg_asm, const int64_t* ctg_boff,
                     const int64_t* ctg_local, int64_t nctg, const int64_t* u, const float* r, float p, int rc_mode, int64_t n,
                     int64_t* asm_index, int64_t* start, uint8_t* rc, int64_t* coords, int32_t* status, void* stream);

/* sample()'s draws and coordinates in one launch, for graphs that replay sample() without torch's generator: the
 * draws are those torch.randint(0, total, (n,)) and (rc_mode 2) torch.rand(n) make on a CUDA generator in this
 * state (the same Philox states, element-to-thread mapping and transforms as torch's kernels for this device), then
 * the arithmetic of pv_sample_coords. rng (device): the generator's seed and Philox offset; the launch advances the
 * offset by what those two torch calls would (pv_torch_draw_geometry's inc_all), so replaying it call after call
 * follows the generator's stream. With rng NULL the state is seed / offset (by value) and the caller advances its
 * generator by inc_all itself. u_out / r_out (device, or NULL): the draws. All pointers device except as noted. */
typedef struct pv_philox {
    uint64_t seed, offset;
    uint32_t arrived, pad;      /* launch bookkeeping: zero between launches */
} pv_philox;
int pv_sample_draw_coords(const int64_t* cum, const int64_t* valid, const int64_t* ctg_asm, const int64_t* ctg_boff,
                          const int64_t* ctg_local, int64_t nctg, uint64_t total, pv_philox* rng, uint64_t seed, uint64_t offset,
                          float p, int rc_mode, int64_t n, int64_t* asm_index, int64_t* start, uint8_t* rc, int64_t* coords,
                          int32_t* status, int64_t* u_out, float* r_out, void* stream);
/* torch's launch for those draws on a device of sm_count SMs and threads_per_sm threads per SM (host, no GPU needed):
 * the grid's threads and the Philox offset the randint call consumes (inc_int) and both calls consume (inc_all) */
int pv_torch_draw_geometry(int64_t n, uint64_t total, int rc_mode, int sm_count, int threads_per_sm, uint64_t* threads,
                           uint64_t* inc_int, uint64_t* inc_all);

/* pv_windows for callers that must not allocate device memory. This entry point has no counterpart in the reference.
 * Some callers cannot call cudaMalloc or hand over a scratch buffer: a data-loading hook inside a training framework
 * whose caching allocator already owns the device memory (a direct cudaMalloc there can fail or fragment its pool),
 * or code that must not stall the device (cudaMalloc / cudaFree can synchronise it). This variant takes the same
 * inputs and outputs as pv_windows but keeps its scratch - the split form's work queue, its plan (the decode results
 * of every item) and list of general-path items, and the block buffers - in a fixed array of PV_NOALLOC_SCRATCH_BYTES that the library places in
 * device memory; every GPU that loads the library holds its own copy of that array until the process exits. A call
 * that would need more scratch than that (pv_windows_work_bytes) returns PV_EARG (message in pv_kernels_last_error())
 * without launching; split it into smaller calls. The first call on a device looks up that device's array address
 * (cudaGetSymbolAddress, with the device current) and keeps it for later calls, so make that first call before any
 * CUDA stream capture; the kept address assumes the device's primary context lives as long as the process (after a
 * cudaDeviceReset, do not call this again). The calls on one device share its array: two calls on the same device
 * that run on the GPU at the same time (on different streams) race on it and must not overlap; calls on different
 * devices use different arrays and may. Nothing in it needs to start at zero: the call's first kernel zeroes the
 * queue, and every byte of the plan, the list and a block buffer is written before it is read. The call makes no cudaMalloc, cudaFree or other allocation. */
#define PV_NOALLOC_SCRATCH_BYTES (16u << 20)
int pv_windows_noalloc(const pv_dev_cohort* cohort, const int64_t* asm_index, const int64_t* start, int64_t n, int64_t W,
                       const uint8_t* rc, int tokens, int apply_case, uint8_t* out, int32_t* status, void* stream);

/* ---- device: the checkpoint index (no counterpart in the reference, whose decoder always starts at a block's start) */

/* bytes of the checkpoint index of a cohort of nblocks pooled blocks at stride 1 << ckpt_shift (0 when the stride is
 * not a power of two between 256 and Q) */
size_t pv_index_bytes(uint32_t Q, uint64_t nblocks, uint32_t ckpt_shift);
/* Decode every block of the cohort once on the device (blocks served from the block cache are skipped) and write its
 * checkpoints into out (pv_index_bytes bytes, 16-byte aligned, device). cohort->ckpt is ignored. *nbad (device uint64,
 * zeroed by the caller, or NULL) counts the blocks that failed. brun (device uint32 [nblocks], or NULL) receives the
 * blocks' first lower-case runs (pv_dev_cohort.brun). cost (device uint16 [nblocks], or NULL) receives each block's
 * decode cost: the largest, over its stride cells, of the events starting in the cell plus the literal bytes decoded
 * in it (the serial work of the block's costliest window item; 0 for a cached or failed block, saturating at 65535).
 * Asynchronous on `stream`. */
int pv_index_build(const pv_dev_cohort* cohort, uint64_t nblocks, uint32_t ckpt_shift, pv_ckpt* out, uint64_t* nbad, uint32_t* brun,
                   uint16_t* cost, void* stream);

/* out[i] = the complement of ref[n - 1 - i] (A <-> T, C <-> G, every other byte as it is), i < n: the reverse-complement
 * reference of pv_dev_cohort.rcref (no counterpart in the reference, which reverses and complements each copied byte).
 * Device pointers; asynchronous on `stream`. */
int pv_rc_reference(const uint8_t* ref, uint64_t n, uint8_t* out, void* stream);

/* ---- device: the whole-assembly checks (Cohort.check_full / fasta, panvram/cohort.py:224-234, whose FASTA rebuild
 * and XXH3 run on the host in the reference, pv_core.cpp:138-176) ---- */

/* One FASTA record (contig) over a decoded base stream: at fasta_off, '>' + the header's hdr_len bytes (at hdr_off in
 * the header blob) + '\n', then bases [boff, boff + len) of the stream in lines of line_width bases, each followed
 * by '\n' (the layout pv_core_fasta_write writes). */
typedef struct pv_fasta_rec {
    uint64_t fasta_off, boff, len, hdr_off;
    uint32_t hdr_len, line_width;
} pv_fasta_rec;
/* A FASTA file described over a device base stream (all pointers device). keys: XXH3's default secret as the device
 * reads it (24 little-endian words, then the last stripe's 8 and the merge's 8 keys; pv_xxh3.h). */
typedef struct pv_fasta_view {
    const pv_fasta_rec* recs; const uint8_t* hdrs; const uint8_t* bases;
    uint64_t nrec, nbases, fasta_len;
    uint64_t keys[40];
} pv_fasta_view;
/* contrib[j nblk + k] (device uint64 [8 nblk], 16-byte aligned) = word j of the sum of XXH3's accumulate steps over the
 * FASTA's 1024-byte block blk0 + k, from zero accumulators: the data-parallel half of XXH3's long-input loop, lane-major
 * (each accumulator's sums contiguous). Blocks must lie wholly inside the FASTA. Asynchronous on `stream`. */
int pv_fasta_xxh3_blocks(const pv_fasta_view* view, uint64_t blk0, uint64_t nblk, uint64_t* contrib, void* stream);
/* out[0 : p1 - p0] (device, 16-byte aligned) = FASTA bytes [p0, p1), p1 <= fasta_len. Asynchronous on `stream`. */
int pv_fasta_bytes(const pv_fasta_view* view, uint64_t p0, uint64_t p1, uint8_t* out, void* stream);
/* Per-block XXH3 of a decoded upper-case base stream (device, 16-byte aligned) against want[] (device uint64 [nb]):
 * *first_bad (a device int64 the caller sets to INT64_MAX) is lowered to the first block that differs. Blocks of 240
 * bases or fewer (only an assembly's last block can be one) are skipped: the caller checks those on the host. */
int pv_block_xxh3_check(const uint8_t* bases, uint64_t nbases, uint32_t Q, const uint64_t* want, const uint64_t* keys40,
                        int64_t* first_bad, void* stream);
/* lower-case runs of assembly asm_index applied in place to its decoded stream on the device (pv_core_apply_case's
 * device twin): the runs as the window kernel reads them from the uploaded cohort; max_runs >= the assembly's run
 * count (pv_asm_info.lower_case_runs) sizes the launch. */
int pv_apply_case_device(const pv_dev_cohort* cohort, int64_t asm_index, uint64_t max_runs, uint8_t* bases, uint64_t nbases,
                         void* stream);

/* assembly asm_index's FASTA layout (host arrays; with recs == NULL only the three sizes): records in file order,
 * header bytes concatenated. A contig with bases and line width 0 is refused (PV_EFORMAT). */
int pv_core_fasta_layout(const pv_core* c, int64_t asm_index, pv_fasta_rec* recs, uint64_t rec_cap, uint8_t* hdrs,
                         uint64_t hdr_cap, uint64_t* nrec, uint64_t* hdr_bytes, uint64_t* fasta_len);
/* the archive's per-block XXH3 values as read at open (a view into the core; NULL and 0 without flag bit 0) */
int pv_core_block_hashes(const pv_core* c, int64_t asm_index, const uint64_t** hashes, uint64_t* n, uint32_t* Q);
/* Host drivers of the above for assembly asm_index of a Core (they upload the record table, run the kernels on
 * `stream` and wait for them). work: device scratch of pv_core_device_check_work_bytes() bytes, 16-byte aligned.
 * pv_core_fasta_xxh3_device: XXH3 of the FASTA rebuilt from a decoded stream with case applied (bases: device), equal
 * to pv_core_fasta_xxh3 of the same stream; the serial scramble chain runs on the host while the device forms the
 * next chunk's block sums (chunk_blocks 1024-byte blocks per round trip, at most and by default (0) 65,536). pv_core_fasta_write_device: the FASTA bytes into out (device, 16-byte aligned; size
 * query with out == NULL). pv_core_check_block_hashes_device: pv_core_check_block_hashes of a device stream. */
size_t pv_core_device_check_work_bytes(const pv_core* c, int64_t asm_index);
int pv_core_fasta_xxh3_device(const pv_core* c, int64_t asm_index, const uint8_t* bases, uint64_t nbases, uint64_t chunk_blocks,
                              void* work, size_t work_bytes, void* stream, uint64_t* out_hash);
int pv_core_fasta_write_device(const pv_core* c, int64_t asm_index, const uint8_t* bases, uint64_t nbases, uint8_t* out,
                               uint64_t cap, void* work, size_t work_bytes, void* stream, uint64_t* size);
int pv_core_check_block_hashes_device(const pv_core* c, int64_t asm_index, const uint8_t* upper_bases, uint64_t nbases,
                                      void* work, size_t work_bytes, void* stream, int64_t* first_bad);
/* XXH3_64bits of a host buffer longer than 240 bytes by the same block sums, scramble chain and finish that the
 * device path splits (host only; it checks that restatement against the xxHash library) */
int pv_xxh3_64_long_host(const void* data, uint64_t len, uint64_t* out_hash);

/* Window coordinates that the caller holds in pinned host memory (asm_host, start_host int64 [n]; rc_host uint8 [n]
 * or NULL; cudaHostAlloc'd), gathered into device arrays by a kernel that reads them through their mapped addresses,
 * ordered on `stream` like a copy. Cohort.windows uses it for pinned host inputs in place of the reference's
 * host-to-device copies (cohort.py:139-141, `.to(device)`): a copy engine busy with other transfers (the previous
 * batch's windows going to the host) does not delay it. The host arrays must stay unchanged until the stream has
 * passed this point. */
int pv_coords_from_host(const int64_t* asm_host, const int64_t* start_host, const uint8_t* rc_host, int64_t n, int64_t* asm_index,
                        int64_t* start, uint8_t* rc, void* stream);

/* The int32 status word read back for Cohort.windows / sample(check=True) (cohort.py:153-156 reads it with
 * status.item()): one thread stores it, after the work queued before it on `stream`, into host_word, which must be
 * pinned host memory (cudaHostAlloc, mapped into the device's address space); the caller then waits for the stream
 * and reads host_word. Unlike a device-to-host copy, this never waits behind other copies in flight (for example the
 * previous batch's windows being copied to the host on another stream). */
int pv_status_to_host(const int32_t* status, int32_t* host_word, void* stream);

/* at most how many kernel launches one pv_windows call with these sizes makes (0 for an empty call; 3 for the split
 * form, 1 for the fused one) */
int pv_windows_launches(int64_t n, int64_t W);
/* the form a pv_windows_ex call with these sizes and flags takes: *launches 1 (pv_windows_kernel) or 3
 * (pv_decode_kernel + pv_emit_kernel + pv_heavy_kernel; *dec_lanes items per decode warp), 0 for an empty call. cell: the cohort's item
 * cell, its checkpoint stride (1 << ckpt_shift) when it has an index, else its block size Q. */
int pv_windows_form(uint32_t cell, int64_t n, int64_t W, uint32_t flags, int* launches, uint32_t* dec_lanes);
/* message of the calling thread's last pv_windows / pv_windows_ex argument or launch failure */
const char* pv_kernels_last_error(void);

#ifdef __cplusplus
}
#endif
