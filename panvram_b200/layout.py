"""Python mirror of csrc/pv_layout.h: the refrel3 model's context alphabets (refrel3.h:29-41) and the offsets of the
per-assembly device decode table. Used by tests to check the table the host builds, slot by slot."""
NCTX, AB, NBIG = 61, 104, 15
C_LL, C_LITR, C_LIT2, C_KIND, C_DELTA, C_REPK, C_REPD, C_DIR, C_SELF, C_LEN, C_FLIPK, C_FLIPD = 0, 4, 14, 31, 47, 49, 50, 51, 52, 53, 59, 60
TAB_CUM8 = 0
TAB_BUCKET = 64
TAB_BIDX = TAB_CUM8 + NCTX * 16
TAB_DOFF = TAB_BIDX + NBIG * (4096 // TAB_BUCKET)
TAB_DENSE = TAB_DOFF + 32
TAB_MAX_BYTES = 8208


def alpha(c):
    if c < C_LITR:
        return AB
    if c < C_DELTA:
        return 6
    if c < C_REPK:
        return AB
    return {C_REPK: 3, C_REPD: AB, C_DIR: 2, C_SELF: AB, C_FLIPK: 4, C_FLIPD: AB}.get(c, AB)


def big_index(c):
    if c < C_LITR:
        return c
    if c < C_DELTA:
        return -1
    if c < C_REPK:
        return 4 + c - C_DELTA
    if c == C_REPD:
        return 6
    if c == C_SELF:
        return 7
    if C_LEN <= c < C_FLIPK:
        return 8 + c - C_LEN
    if c == C_FLIPD:
        return 14
    return -1


ALPHA = [alpha(c) for c in range(NCTX)]
