// pv_host.cpp - panvram_b200 host side: the reference FASTA (upper-cased, SHA-256), refrel3 v1 archives opened with
// every FORMAT section-5 check, and the cohort pooled into the device layout of pv_layout.h (the C ABI of
// include/panvram_b200.h). Replaces the reference's pv_v1.h reader (open_v1, pv_v1.h:99-146) and its Core
// (pv_core.cpp:23-183): same checks in the same order, same refusal text, one block size per cohort.
//
// Open reads each archive's header and meta section first (every check runs before any payload is read) and then
// reads every payload straight into its place in the pooled buffer, on `threads` host threads.
#include <fcntl.h>
#include <openssl/sha.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <cstdio>
#include <cstring>
#include <memory>
#include <mutex>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

#include "pv_layout.h"

// runtime-library prototypes (the image ships libzstd.so.1 and libxxhash.so.0 without their headers)
extern "C" {
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
}

namespace {

thread_local std::string g_err;
struct Err : std::runtime_error { using std::runtime_error::runtime_error; };

int fail_with(int code, const std::string& msg) { g_err = msg; return code; }

uint64_t rd64(const uint8_t* p) { uint64_t v; memcpy(&v, p, 8); return v; }
uint32_t rd32(const uint8_t* p) { uint32_t v; memcpy(&v, p, 4); return v; }
std::string hex(const uint8_t* p, size_t n) {
    static const char* d = "0123456789abcdef";
    std::string s;
    for (size_t i = 0; i < n; i++) { s += d[p[i] >> 4]; s += d[p[i] & 15]; }
    return s;
}

template <class F> void parallel_for(uint64_t n, int T, F&& f) {
    if (!n) return;
    T = (int)std::max<uint64_t>(1, std::min<uint64_t>((uint64_t)std::max(1, T), n));
    std::atomic<uint64_t> next{0};
    std::vector<std::thread> th;
    for (int t = 0; t < T; t++) th.emplace_back([&] { for (;;) { const uint64_t i = next.fetch_add(1); if (i >= n) break; f(i); } });
    for (auto& x : th) x.join();
}
int default_threads() { const unsigned h = std::thread::hardware_concurrency(); return h ? (int)h : 4; }

struct File {
    int fd = -1; uint64_t size = 0;
    explicit File(const std::string& p) {
        fd = ::open(p.c_str(), O_RDONLY);
        if (fd < 0) throw Err(p + ": cannot open");
        struct stat st;
        if (fstat(fd, &st)) { ::close(fd); throw Err(p + ": cannot open"); }
        size = (uint64_t)st.st_size;
    }
    ~File() { if (fd >= 0) ::close(fd); }
    bool read_at(uint8_t* dst, uint64_t n, uint64_t off) const {
        while (n) {
            const ssize_t r = ::pread(fd, dst, n > (1u << 30) ? (1u << 30) : n, (off_t)off);
            if (r <= 0) return false;
            dst += r; n -= (uint64_t)r; off += (uint64_t)r;
        }
        return true;
    }
};

// pv_v1.h:42-53: FASTA -> its bases in place (headers and line ends dropped, a..z upper-cased)
uint64_t fasta_bases_inplace(uint8_t* buf, uint64_t n, const std::string& path) {
    if (!n || buf[0] != '>') throw Err(path + ": not FASTA (no header at byte 0)");
    uint64_t i = 0, w = 0;
    while (i < n) {
        if (buf[i] == '>') {
            const uint8_t* e = (const uint8_t*)memchr(buf + i, '\n', n - i);
            if (!e) throw Err(path + ": header without line end");
            i = (uint64_t)(e - buf) + 1;
            continue;
        }
        const uint8_t* e = (const uint8_t*)memchr(buf + i, '\n', n - i);
        if (!e) throw Err(path + ": no final line end");
        const uint64_t le = (uint64_t)(e - buf);
        for (uint64_t k = i; k < le; k++) { const uint8_t c = buf[k]; buf[w++] = (c >= 'a' && c <= 'z') ? (uint8_t)(c - 32) : c; }
        i = le + 1;
    }
    return w;
}

struct Contig { std::string hdr, name; uint64_t len = 0, boff = 0; uint32_t lw = 0; };

struct Arc {
    std::string path, refname;
    uint32_t Q = 0, flags = 0;
    uint64_t nbases = 0, nb = 0, fasta_xxh = 0, bases_xxh = 0, file_bytes = 0, payload_bytes = 0, payload_at = 0;
    std::vector<Contig> rec;
    std::vector<uint64_t> low_s, low_l, hashes;
    std::vector<uint16_t> freq;            // [61][104]
    std::vector<uint32_t> off;             // [nb + 1] payload offsets within the archive's payload
    std::vector<int64_t> st;               // [nb] packed start states c << 1 | dir
    std::vector<uint8_t> tab;              // device decode table (pv_layout.h)
};

std::vector<uint8_t> build_table(const uint16_t* freq);

// pv_v1.h:99-146, every check in the reference's order and with its text; the payload itself is not read here
void open_archive(const std::string& path, const uint8_t ref_sha[32], uint64_t ref_n, Arc& X) {
    File f(path);
    const uint64_t n = f.size;
    auto refuse = [&](const char* w) { throw Err(path + ": refused: " + w); };
    if (n < 136 + 2) refuse("short file");
    std::vector<uint8_t> h(138);
    if (!f.read_at(h.data(), 138, 0)) throw Err(path + ": short read");
    const uint8_t* a = h.data();
    if (memcmp(a, "RFRL3V1\0", 8)) refuse("magic (not refrel3 v1)");
    if (rd32(a + 8) != 1) refuse("version");
    X.Q = rd32(a + 12);
    if (!(X.Q == 1024 || X.Q == 2048 || X.Q == 4096 || X.Q == 16384)) refuse("block size");
    X.flags = rd32(a + 16);
    if (X.flags & ~1u) refuse("unknown flags");
    if (rd32(a + 20)) refuse("reserved");
    X.nbases = rd64(a + 64); X.nb = rd64(a + 72); X.fasta_xxh = rd64(a + 80); X.bases_xxh = rd64(a + 88);
    const uint64_t mz = rd64(a + 96), mr = rd64(a + 104), hs = rd64(a + 112), pl = rd64(a + 120);
    const uint16_t nl = (uint16_t)(a[136] | a[137] << 8);
    const uint64_t pstart = 136ull + 2 + nl + mz + hs;
    if (mz > n || hs > n || pl > n || pstart > n || pstart + pl != n) refuse("section sizes");
    if (X.nb != (X.nbases + X.Q - 1) / X.Q || (X.nbases && !X.nb)) refuse("block count");
    if (hs != ((X.flags & 1u) ? X.nb * 8 : 0)) refuse("hash section size");
    h.resize(pstart);
    if (!f.read_at(h.data(), pstart, 0)) throw Err(path + ": short read");
    a = h.data();
    {
        const uint64_t want = rd64(a + 128);
        memset(&h[128], 0, 8);
        const uint64_t got = XXH3_64bits(h.data(), pstart);
        memcpy(&h[128], &want, 8);
        if (got != want) refuse("header XXH3");
    }
    if (memcmp(a + 24, ref_sha, 32) || rd64(a + 56) != ref_n) refuse("reference SHA-256 / size differs (wrong reference)");
    X.refname.assign((const char*)a + 138, nl);
    const uint8_t* mzp = a + 138 + nl;
    if (mr > (1ull << 32) || ZSTD_getFrameContentSize(mzp, mz) != mr) refuse("meta frame");
    if (ZSTD_findFrameCompressedSize(mzp, mz) != mz) refuse("meta frame count (exactly one zstd frame)");
    std::vector<uint8_t> M(mr);
    if (ZSTD_decompress(M.data(), mr, mzp, mz) != mr) refuse("meta decompress");
    size_t i = 0; bool bad = false;
    auto need = [&](size_t k) { if (i + k > M.size()) { bad = true; return false; } return true; };
    auto g64 = [&]() -> uint64_t { if (!need(8)) return 0; const uint64_t v = rd64(&M[i]); i += 8; return v; };
    auto g32 = [&]() -> uint32_t { if (!need(4)) return 0; const uint32_t v = rd32(&M[i]); i += 4; return v; };
    auto gl = [&]() -> uint64_t {
        uint64_t v = 0; int sh = 0;
        for (;;) {
            if (!need(1) || sh > 63) { bad = true; return 0; }
            const uint8_t c = M[i++];
            v |= (uint64_t)(c & 0x7F) << sh;
            if (!(c & 0x80)) break;
            sh += 7;
        }
        return v;
    };
    const uint32_t nr = g32();
    uint64_t bo = 0;
    if (nr > M.size()) refuse("records");
    for (uint32_t r = 0; r < nr && !bad; r++) {
        Contig q;
        const uint32_t hl = g32();
        if (!need(hl)) break;
        q.hdr.assign((const char*)&M[i], hl); i += hl;
        q.len = g64(); q.lw = g32();
        if (!q.lw && q.len) bad = true;
        q.name = q.hdr.substr(0, q.hdr.find_first_of(" \t"));
        q.boff = bo; bo += q.len;
        X.rec.push_back(std::move(q));
    }
    if (bad || bo != X.nbases) refuse("contig table");
    const uint64_t nlw = g64();
    uint64_t lst = 0;
    if (nlw > X.nbases) refuse("case runs");
    for (uint64_t k = 0; k < nlw && !bad; k++) {
        const uint64_t g = gl(), l = gl();
        if (lst + g + l > X.nbases) { bad = true; break; }
        X.low_s.push_back(lst + g); X.low_l.push_back(l); lst += g + l;
    }
    if (bad) refuse("case runs");
    X.freq.assign((size_t)pvb::NCTX * pvb::AB, 0);
    for (int c = 0; c < pvb::NCTX && !bad; c++) {
        uint64_t sum = 0;
        for (int s = 0; s < pvb::alpha(c); s++) {
            const uint64_t fv = gl();
            if (fv > pvb::MTOT) bad = true;
            X.freq[(size_t)c * pvb::AB + s] = (uint16_t)fv;
            sum += fv;
        }
        if (sum && sum != pvb::MTOT) bad = true;
    }
    if (bad) refuse("model tables");
    X.tab = build_table(X.freq.data());
    if (pl >= (1ull << 32)) refuse("payload over 4 GiB (pooled offsets are 32-bit)");
    X.off.assign(X.nb + 1, 0); X.st.assign(X.nb, 0);
    uint64_t prevc = 0; uint32_t prevd = 0, acc = 0;
    for (uint64_t b = 0; b < X.nb && !bad; b++) {
        const uint64_t len = gl();
        if (len > pl - acc) { bad = true; break; }
        acc += (uint32_t)len; X.off[b + 1] = acc;
        const uint64_t v = gl();
        const int64_t pred = b == 0 ? 0 : (int64_t)(prevd ? prevc - X.Q : prevc + X.Q);
        const uint64_t q = v >> 1;
        const uint32_t dir = (uint32_t)(v & 1);
        const uint64_t c = (uint64_t)(pred + ((int64_t)(q >> 1) ^ -(int64_t)(q & 1)));
        X.st[b] = (int64_t)(c << 1) | (int64_t)dir;           // as pack_state (pv_v1.h:96)
        prevc = c; prevd = dir;
    }
    if (bad || i != M.size() || acc != pl) refuse("block table");
    if (X.flags & 1u) { X.hashes.resize(X.nb); memcpy(X.hashes.data(), a + 138 + nl + mz, X.nb * 8); }
    X.payload_bytes = pl; X.payload_at = pstart; X.file_bytes = n; X.path = path;
}

// the per-assembly decode table of pv_layout.h from the model frequencies (its size is a multiple of 16)
std::vector<uint8_t> build_table(const uint16_t* freq) {
    std::vector<uint8_t> out((size_t)pvb::TAB_MAX, 0);
    uint16_t* cum8 = (uint16_t*)(out.data() + pvb::TAB_CUM8);
    uint8_t* bidx = out.data() + pvb::TAB_BIDX;
    uint16_t* doff = (uint16_t*)(out.data() + pvb::TAB_DOFF);
    uint32_t* dense = (uint32_t*)(out.data() + pvb::TAB_DENSE);
    uint32_t nd = 0;
    for (int c = 0; c < pvb::NCTX; c++) {
        const int A = pvb::alpha(c);
        const uint16_t* f = freq + (size_t)c * pvb::AB;
        uint32_t cum[pvb::AB + 1]; cum[0] = 0;
        for (int s = 0; s < A; s++) cum[s + 1] = cum[s] + f[s];
        const int bi = pvb::big_index(c);
        if (bi < 0) {
            for (int k = 0; k < 8; k++) cum8[c * 8 + k] = (uint16_t)cum[std::min(k, A)];
            continue;
        }
        doff[bi] = (uint16_t)nd;
        uint32_t* d = dense + nd;
        int nu = 0;
        for (int s = 0; s < A; s++) if (f[s]) d[nu++] = pvb::dense_entry(cum[s], f[s], (uint32_t)s);
        if (!nu) d[nu++] = 0;                                  // an unused context: one zero-frequency entry
        uint8_t* bx = bidx + bi * (4096 / pvb::TAB_BUCKET);
        int u = 0;
        for (int k = 0; k < 4096 / pvb::TAB_BUCKET; k++) {
            const uint32_t slot = (uint32_t)k * pvb::TAB_BUCKET;
            while (u + 1 < nu && slot >= pvb::dense_cum(d[u]) + pvb::dense_freq(d[u])) u++;
            bx[k] = (uint8_t)u;
        }
        nd += (uint32_t)nu;
    }
    doff[pvb::NBIG] = (uint16_t)nd;
    out.resize(((size_t)pvb::TAB_DENSE + 4 * nd + 15) & ~(size_t)15);
    return out;
}

uint64_t fasta_size(const Arc& X) {
    uint64_t size = 0;
    for (auto& r : X.rec) size += 2 + r.hdr.size() + r.len + (r.lw ? (r.len + r.lw - 1) / r.lw : 0);
    return size;
}

}  // namespace

struct pv_core {
    std::string ref_path;
    uint8_t ref_sha[32] = {0};
    uint64_t ref_n = 0;
    std::vector<uint8_t> ref;              // 64 B zero | bases | 64 B zero
    std::vector<Arc> A;
    uint32_t Q = 0;
    int threads = 0;
    // pooled, in the device layout
    std::vector<uint8_t> payload;
    std::vector<uint64_t> blocks, low;
    std::vector<pv_asm_rec> asms;
    std::vector<uint8_t> tabs;
    uint64_t tab_max = 0;
    std::vector<int64_t> ctg_asm, ctg_local, ctg_boff, ctg_len;
    // opt-in compact forms (pv_compact.h): then `ref` / `blocks` are empty
    bool packed = false, compact = false;
    std::vector<uint32_t> pref, pidx;
    std::vector<pv_ref_run> pruns;
    std::vector<pv_blk_group> groups;
    std::vector<uint32_t> btab;
    std::vector<int64_t> bexc;
};

namespace {
void load_reference(pv_core& C, const std::string& path) {
    File f(path);
    const uint64_t s = f.size;
    C.ref.assign(64 + s + 64, 0);
    if (!f.read_at(C.ref.data() + 64, s, 0)) throw Err(path + ": short read");
    C.ref_n = fasta_bases_inplace(C.ref.data() + 64, s, path);
    memset(C.ref.data() + 64 + C.ref_n, 0, 64);
    C.ref.resize(64 + C.ref_n + 64);
    C.ref.shrink_to_fit();
    SHA256(C.ref.data() + 64, C.ref_n, C.ref_sha);
}

// The reference in 2 bits per base plus its runs of other bytes (the reference's PackedRef, pv_compact.h:19-28, built
// like pv_core.cpp:52-62), then the byte copy is dropped. Words are packed in parallel chunks; runs are collected per
// chunk and joined where a run crosses a chunk boundary.
void pack_reference(pv_core& C) {
    const uint64_t n = C.ref_n, nw = (n + 15) / 16;
    const uint8_t* R = C.ref.data() + 64;
    C.pref.assign(nw + 4, 0);
    const uint64_t chunk_words = 1u << 20;
    const uint64_t nchunks = (nw + chunk_words - 1) / chunk_words;
    std::vector<std::vector<pv_ref_run>> part(std::max<uint64_t>(1, nchunks));
    parallel_for(nchunks, C.threads, [&](uint64_t t) {
        const uint64_t q0 = t * chunk_words * 16, q1 = std::min(n, q0 + chunk_words * 16);
        std::vector<pv_ref_run>& runs = part[t];
        for (uint64_t q = q0; q < q1; q++) {
            const uint8_t b = R[q];
            const uint32_t code = b == 'A' ? 0 : b == 'C' ? 1 : b == 'G' ? 2 : b == 'T' ? 3 : 4;
            if (code < 4) { C.pref[q >> 4] |= code << ((q & 15) * 2); continue; }
            if (!runs.empty() && runs.back().byte == b && runs.back().start + runs.back().len == q) runs.back().len++;
            else runs.push_back(pv_ref_run{q, 1, b});
        }
    });
    C.pruns.clear();
    for (auto& runs : part)
        for (const pv_ref_run& r : runs) {
            if (!C.pruns.empty() && C.pruns.back().byte == r.byte && C.pruns.back().start + C.pruns.back().len == r.start) C.pruns.back().len += r.len;
            else C.pruns.push_back(r);
        }
    const uint64_t nreal = C.pruns.size();
    C.pruns.push_back(pv_ref_run{~0ull, 0, 0});       // sentinel: every scan stops at it without a bound check
    const uint64_t nbk = (n >> PV_REF_BUCKET_SHIFT) + 2;
    C.pidx.assign(nbk, 0);
    uint64_t i = 0;
    for (uint64_t k = 0; k < nbk; k++) {
        const uint64_t x = k << PV_REF_BUCKET_SHIFT;
        while (i < nreal && C.pruns[i].start + C.pruns[i].len <= x) i++;
        C.pidx[k] = (uint32_t)i;
    }
    if (C.pruns.size() >= (1ull << 32)) throw Err("reference with 2^32 runs of non-ACGT bytes: not packable");
    std::vector<uint8_t>().swap(C.ref);
}

// The compact block table of one assembly (the reference's CompactTab, pv_compact.h:30-46, built like
// pv_core.cpp:92-111): groups of PV_BLK_GROUP blocks, 32 bits per block, exception states in block order.
void compact_blocks(pv_core& C, const Arc& X, uint64_t pay_base, uint64_t blk_base, uint64_t grp_base, std::vector<int64_t>& exc) {
    const int64_t Q = (int64_t)C.Q;
    for (uint64_t b = 0; b < X.nb; b++) {
        const uint64_t len = (uint64_t)(X.off[b + 1] - X.off[b]);
        if (len > 65535) throw Err(X.path + ": block payload over 65535 B - open without compact_blocks");
        pv_blk_group& G = C.groups[grp_base + b / PV_BLK_GROUP];
        const uint32_t k = (uint32_t)(b % PV_BLK_GROUP);
        int32_t code = 0;
        if (k == 0) {
            G.off = pay_base + X.off[b]; G.state = X.st[b]; G.exc_mask = 0; G.exc_base = 0; G.cache_mask = 0; G.cache_base = 0;
        } else {
            const int64_t prev = X.st[b - 1], pc = prev >> 1;
            const int64_t pred = (prev & 1) ? pc - Q : pc + Q;
            const int64_t delta = (X.st[b] >> 1) - pred;
            if (delta >= -16383 && delta <= 16383) code = (int32_t)(delta * 2 + (X.st[b] & 1));
            else { code = PV_CODE_EXC; G.exc_mask |= 1u << k; exc.push_back(X.st[b]); }
        }
        C.btab[blk_base + b] = (uint32_t)len | ((uint32_t)(uint16_t)(int16_t)code << 16);
    }
}

void pool(pv_core& C, const std::vector<std::string>& paths) {
    const size_t n = C.A.size();
    std::vector<uint64_t> pb(n), bb(n), lb(n), cb(n), tb(n), gb(n);
    uint64_t sp = 0, sb = 0, sl = 0, sc = 0, st = 0, sg = 0;
    for (size_t i = 0; i < n; i++) {
        pb[i] = sp; bb[i] = sb; lb[i] = sl; cb[i] = sc; tb[i] = st; gb[i] = sg;
        sp += C.A[i].payload_bytes; sb += C.A[i].nb; sl += C.A[i].low_s.size(); sc += C.A[i].rec.size(); st += C.A[i].tab.size();
        sg += (C.A[i].nb + PV_BLK_GROUP - 1) / PV_BLK_GROUP;
        C.tab_max = std::max<uint64_t>(C.tab_max, C.A[i].tab.size());
    }
    C.payload.assign(sp + 64, 0);
    std::vector<std::vector<int64_t>> exc(n);
    if (C.compact) {
        C.groups.assign(std::max<uint64_t>(1, sg), pv_blk_group{});
        C.btab.assign(std::max<uint64_t>(1, sb) + PV_BLK_GROUP, 0);      // a warp reads a whole group past the last block
    } else {
        C.blocks.assign(2 * std::max<uint64_t>(1, sb), 0);
    }
    C.low.assign(2 * std::max<uint64_t>(1, sl), 0);
    C.asms.assign(n, pv_asm_rec{});
    C.tabs.assign(st + 16, 0);                            // (16 zero bytes after the last table: a lookup may read one entry ahead)
    C.ctg_asm.assign(sc, 0); C.ctg_local.assign(sc, 0); C.ctg_boff.assign(sc, 0); C.ctg_len.assign(sc, 0);
    std::mutex mu; std::string first;
    parallel_for(n, C.threads, [&](uint64_t i) {
        try {
            Arc& X = C.A[i];
            File f(paths[i]);
            if (f.size != X.file_bytes || !f.read_at(C.payload.data() + pb[i], X.payload_bytes, X.payload_at))
                throw Err(X.path + ": short read");
            if (C.compact) {
                compact_blocks(C, X, pb[i], bb[i], gb[i], exc[i]);
            } else {
                for (uint64_t b = 0; b < X.nb; b++) {
                    C.blocks[2 * (bb[i] + b)] = pvb::block_loc(pb[i] + X.off[b], (uint64_t)(X.off[b + 1] - X.off[b]));
                    C.blocks[2 * (bb[i] + b) + 1] = (uint64_t)X.st[b];
                }
            }
            pv_asm_rec& r = C.asms[i];
            r.nbases = X.nbases; r.blk_base = bb[i]; r.nb = X.nb; r.low_base = lb[i]; r.low_cnt = X.low_s.size();
            r.tab_off = tb[i]; r.tab_bytes = X.tab.size(); r.grp_base = gb[i];
            for (size_t k = 0; k < X.low_s.size(); k++) { C.low[2 * (lb[i] + k)] = X.low_s[k]; C.low[2 * (lb[i] + k) + 1] = X.low_s[k] + X.low_l[k]; }
            memcpy(C.tabs.data() + tb[i], X.tab.data(), X.tab.size());
            for (size_t k = 0; k < X.rec.size(); k++) {
                C.ctg_asm[cb[i] + k] = (int64_t)i; C.ctg_local[cb[i] + k] = (int64_t)k;
                C.ctg_boff[cb[i] + k] = (int64_t)X.rec[k].boff; C.ctg_len[cb[i] + k] = (int64_t)X.rec[k].len;
            }
            std::vector<uint32_t>().swap(X.off); std::vector<int64_t>().swap(X.st); std::vector<uint8_t>().swap(X.tab);
        } catch (const std::exception& e) {
            std::lock_guard<std::mutex> g(mu);
            if (first.empty()) first = e.what();
        }
    });
    if (!first.empty()) throw Err(first);
    if (C.compact) {                                  // exception states pooled in block order, group bases after
        uint64_t e = 0;
        for (size_t i = 0; i < n; i++) {
            const uint64_t ng = (C.A[i].nb + PV_BLK_GROUP - 1) / PV_BLK_GROUP;
            for (uint64_t g = 0; g < ng; g++) {
                C.groups[gb[i] + g].exc_base = (uint32_t)e;
                e += (uint64_t)__builtin_popcount(C.groups[gb[i] + g].exc_mask);
            }
            C.bexc.insert(C.bexc.end(), exc[i].begin(), exc[i].end());
        }
        if (C.bexc.size() >= (1ull << 32)) throw Err("more than 2^32 block-state exceptions: open without compact_blocks");
        if (C.bexc.empty()) C.bexc.push_back(0);
    }
}

const Arc* arc_at(const pv_core* c, int64_t i) {
    if (!c || i < 0 || i >= (int64_t)c->A.size()) { g_err = "assembly index out of range"; return nullptr; }
    return &c->A[(size_t)i];
}
void copy_str(const std::string& s, char* out, size_t cap) {
    if (!out || !cap) return;
    const size_t k = std::min(cap - 1, s.size());
    memcpy(out, s.data(), k); out[k] = 0;
}
}  // namespace

extern "C" {

const char* pv_last_error(void) { return g_err.c_str(); }

int pv_core_open(const char* reference, const char* const* paths, int64_t npaths, int threads, int packed_reference,
                 int compact_blocks, pv_core** out) {
    *out = nullptr;
    std::unique_ptr<pv_core> C(new pv_core());
    C->packed = packed_reference != 0;
    C->compact = compact_blocks != 0;
    try {
        if (npaths <= 0) throw Err("no archives");
        C->ref_path = reference;
        C->threads = threads > 0 ? threads : default_threads();
        load_reference(*C, reference);
        if (C->ref_n >= (1ull << 32)) throw Err("reference of 2^32 bases or more: the queue kernel's copy positions are 32-bit");
        std::vector<std::string> ps(paths, paths + npaths);
        C->A.resize(ps.size());
        std::mutex mu; std::string first;
        parallel_for(ps.size(), C->threads, [&](uint64_t i) {
            try { open_archive(ps[i], C->ref_sha, C->ref_n, C->A[i]); }
            catch (const std::exception& e) { std::lock_guard<std::mutex> g(mu); if (first.empty()) first = e.what(); }
        });
        if (!first.empty()) throw Err(first);
        C->Q = C->A[0].Q;
        for (auto& x : C->A)
            if (x.Q != C->Q)
                throw Err(x.path + ": block size " + std::to_string(x.Q) + " differs from " + std::to_string(C->Q) + " (one dataset per cohort)");
        pool(*C, ps);
        if (C->packed) pack_reference(*C);
    } catch (const Err& e) {
        return fail_with(PV_EFORMAT, e.what());
    } catch (const std::bad_alloc&) {
        return fail_with(PV_EIO, "out of host memory while opening the cohort");
    }
    *out = C.release();
    return PV_OK;
}

void pv_core_free(pv_core* c) { delete c; }
int64_t pv_core_n(const pv_core* c) { return (int64_t)c->A.size(); }
uint32_t pv_core_q(const pv_core* c) { return c->Q; }
uint64_t pv_core_ref_bases(const pv_core* c) { return c->ref_n; }
void pv_core_ref_sha256(const pv_core* c, char out[65]) { const std::string h = hex(c->ref_sha, 32); memcpy(out, h.c_str(), 65); }

void pv_core_release_uploaded(pv_core* c) {
    if (!c) return;
    std::vector<uint8_t>().swap(c->ref);
    std::vector<uint8_t>().swap(c->payload);
    std::vector<uint32_t>().swap(c->pref);
}

int pv_core_pools(const pv_core* c, pv_host_pools* o) {
    o->ref_padded = c->ref.data(); o->ref_padded_bytes = c->ref.size();
    o->payload = c->payload.data(); o->payload_bytes = c->payload.size();
    o->blocks = c->blocks.data(); o->blocks_bytes = c->blocks.size() * 8;
    o->asms = c->asms.data(); o->asms_bytes = c->asms.size() * sizeof(pv_asm_rec);
    o->tabs = c->tabs.data(); o->tabs_bytes = c->tabs.size(); o->tab_max = c->tab_max;
    o->low = c->low.data(); o->low_bytes = c->low.size() * 8;
    o->ctg_asm = c->ctg_asm.data(); o->ctg_local = c->ctg_local.data(); o->ctg_boff = c->ctg_boff.data(); o->ctg_len = c->ctg_len.data();
    o->ncontigs = c->ctg_asm.size();
    o->pref = c->pref.data(); o->pref_bytes = c->pref.size() * 4;
    o->pruns = c->pruns.data(); o->pruns_bytes = c->pruns.size() * sizeof(pv_ref_run); o->pnruns = c->pruns.empty() ? 0 : c->pruns.size() - 1;
    o->pidx = c->pidx.data(); o->pidx_bytes = c->pidx.size() * 4;
    o->groups = c->groups.data(); o->groups_bytes = c->groups.size() * sizeof(pv_blk_group);
    o->btab = c->btab.data(); o->btab_bytes = c->btab.size() * 4;
    o->bexc = c->bexc.data(); o->bexc_bytes = c->bexc.size() * 8;
    o->packed = c->packed; o->compact = c->compact;
    if (c->packed) { o->ref_padded = nullptr; o->ref_padded_bytes = 0; }
    if (c->compact) { o->blocks = nullptr; o->blocks_bytes = 0; }
    return PV_OK;
}

int pv_core_info(const pv_core* c, int64_t i, pv_asm_info* o) {
    const Arc* X = arc_at(c, i);
    if (!X) return PV_EARG;
    o->Q = X->Q; o->block_hashes = !X->hashes.empty();
    o->bases = X->nbases; o->blocks = X->nb; o->file_bytes = X->file_bytes; o->payload_bytes = X->payload_bytes;
    o->contigs = X->rec.size(); o->lower_case_runs = X->low_s.size(); o->fasta_xxh3 = X->fasta_xxh; o->bases_xxh3 = X->bases_xxh;
    return PV_OK;
}
int pv_core_info_strings(const pv_core* c, int64_t i, char* path, size_t path_cap, char* refname, size_t ref_cap) {
    const Arc* X = arc_at(c, i);
    if (!X) return PV_EARG;
    copy_str(X->path, path, path_cap); copy_str(X->refname, refname, ref_cap);
    return PV_OK;
}
int64_t pv_core_ncontigs(const pv_core* c, int64_t i) { const Arc* X = arc_at(c, i); return X ? (int64_t)X->rec.size() : -1; }
int pv_core_contig(const pv_core* c, int64_t i, int64_t k, char* hdr, size_t hdr_cap, char* name, size_t name_cap, uint64_t* len,
                   uint64_t* boff, uint32_t* lw) {
    const Arc* X = arc_at(c, i);
    if (!X) return PV_EARG;
    if (k < 0 || k >= (int64_t)X->rec.size()) return fail_with(PV_EARG, "contig index out of range");
    const Contig& r = X->rec[(size_t)k];
    copy_str(r.hdr, hdr, hdr_cap); copy_str(r.name, name, name_cap);
    *len = r.len; *boff = r.boff; *lw = r.lw;
    return PV_OK;
}

int pv_core_fasta_xxh3(const pv_core* c, int64_t i, const uint8_t* B, uint64_t nbases, uint64_t* out_hash) {
    const Arc* X = arc_at(c, i);
    if (!X) return PV_EARG;
    if (nbases != X->nbases) return fail_with(PV_EARG, "bases: uint8 CPU tensor of the assembly's length");
    XXH3_state_t* h = XXH3_createState();
    XXH3_64bits_reset(h);
    std::vector<char> buf; buf.reserve(1 << 21);
    auto flush = [&](bool all) { if (all || buf.size() >= (1u << 20)) { XXH3_64bits_update(h, buf.data(), buf.size()); buf.clear(); } };
    for (auto& r : X->rec) {
        buf.push_back('>'); buf.insert(buf.end(), r.hdr.begin(), r.hdr.end()); buf.push_back('\n');
        for (uint64_t x = 0; x < r.len; x += r.lw) {
            const uint64_t k = std::min<uint64_t>(r.lw, r.len - x);
            buf.insert(buf.end(), B + r.boff + x, B + r.boff + x + k); buf.push_back('\n');
            flush(false);
        }
    }
    flush(true);
    *out_hash = XXH3_64bits_digest(h);
    XXH3_freeState(h);
    return PV_OK;
}

int pv_core_fasta_write(const pv_core* c, int64_t i, const uint8_t* B, uint64_t nbases, uint8_t* out, uint64_t cap, uint64_t* size) {
    const Arc* X = arc_at(c, i);
    if (!X) return PV_EARG;
    const uint64_t sz = fasta_size(*X);
    *size = sz;
    if (!out) return PV_OK;
    if (nbases != X->nbases || cap < sz) return fail_with(PV_EARG, "FASTA rebuild: base stream or buffer size");
    uint8_t* p = out;
    for (auto& r : X->rec) {
        *p++ = '>'; memcpy(p, r.hdr.data(), r.hdr.size()); p += r.hdr.size(); *p++ = '\n';
        for (uint64_t x = 0; x < r.len; x += r.lw) {
            const uint64_t k = std::min<uint64_t>(r.lw, r.len - x);
            memcpy(p, B + r.boff + x, k); p += k; *p++ = '\n';
        }
    }
    if ((uint64_t)(p - out) != sz) return fail_with(PV_EFORMAT, X->path + ": FASTA size");
    return PV_OK;
}

int pv_core_fasta_layout(const pv_core* c, int64_t i, pv_fasta_rec* recs, uint64_t rec_cap, uint8_t* hdrs, uint64_t hdr_cap,
                         uint64_t* nrec, uint64_t* hdr_bytes, uint64_t* fasta_len) {
    const Arc* X = arc_at(c, i);
    if (!X) return PV_EARG;
    uint64_t fo = 0, ho = 0;
    for (auto& r : X->rec) {
        if (r.len && !r.lw) return fail_with(PV_EFORMAT, X->path + ": contig with bases and line width 0");
        if (recs && ho + r.hdr.size() <= hdr_cap && (uint64_t)(&r - X->rec.data()) < rec_cap) {
            pv_fasta_rec& o = recs[&r - X->rec.data()];
            o.fasta_off = fo; o.boff = r.boff; o.len = r.len; o.hdr_off = ho; o.hdr_len = (uint32_t)r.hdr.size(); o.line_width = r.lw;
            memcpy(hdrs + ho, r.hdr.data(), r.hdr.size());
        } else if (recs) {
            return fail_with(PV_EARG, "FASTA layout: arrays too small");
        }
        fo += 2 + r.hdr.size() + r.len + (r.lw ? (r.len + r.lw - 1) / r.lw : 0);
        ho += r.hdr.size();
    }
    *nrec = X->rec.size(); *hdr_bytes = ho; *fasta_len = fo;
    return PV_OK;
}

int pv_core_block_hashes(const pv_core* c, int64_t i, const uint64_t** hashes, uint64_t* n, uint32_t* Q) {
    const Arc* X = arc_at(c, i);
    if (!X) return PV_EARG;
    *hashes = X->hashes.empty() ? nullptr : X->hashes.data();
    *n = X->hashes.size();
    *Q = X->Q;
    return PV_OK;
}

int pv_core_check_block_hashes(const pv_core* c, int64_t i, const uint8_t* B, uint64_t nbases, int64_t* first_bad) {
    const Arc* X = arc_at(c, i);
    if (!X) return PV_EARG;
    *first_bad = -1;
    if (nbases != X->nbases) return fail_with(PV_EARG, "block hashes: base stream size");
    if (X->hashes.empty()) return PV_OK;
    std::atomic<int64_t> bad{INT64_MAX};
    parallel_for(X->nb, c->threads, [&](uint64_t b) {
        const uint64_t blen = std::min<uint64_t>(X->Q, X->nbases - b * X->Q);
        if (XXH3_64bits(B + b * X->Q, blen) != X->hashes[b]) {
            int64_t cur = bad.load();
            while ((int64_t)b < cur && !bad.compare_exchange_weak(cur, (int64_t)b)) {}
        }
    });
    if (bad.load() != INT64_MAX) *first_bad = bad.load();
    return PV_OK;
}

int pv_core_apply_case(const pv_core* c, int64_t i, uint8_t* B, uint64_t nbases) {
    const Arc* X = arc_at(c, i);
    if (!X) return PV_EARG;
    if (nbases != X->nbases) return fail_with(PV_EARG, "apply_case: base stream size");
    for (size_t r = 0; r < X->low_s.size(); r++)
        for (uint64_t x = X->low_s[r]; x < X->low_s[r] + X->low_l[r]; x++) B[x] |= 0x20;
    return PV_OK;
}

int pv_sha256_file_bases(const char* path, char out[65]) {
    try {
        File f(path);
        std::vector<uint8_t> b(f.size);
        if (!f.read_at(b.data(), f.size, 0)) throw Err(std::string(path) + ": short read");
        const uint64_t n = fasta_bases_inplace(b.data(), b.size(), path);
        uint8_t s[32];
        SHA256(b.data(), n, s);
        const std::string h = hex(s, 32);
        memcpy(out, h.c_str(), 65);
    } catch (const Err& e) {
        return fail_with(PV_EFORMAT, e.what());
    }
    return PV_OK;
}

}  // extern "C"
