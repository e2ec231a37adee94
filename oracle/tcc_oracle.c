/*
 * tcc_oracle.c -- CPU restatement of the tcc graph-aggregation path.
 *
 * TEST INFRASTRUCTURE ONLY (see tcc_oracle.h): the checker for tcc_b200's CUDA
 * path, used by tests/, __graft_entry__.smoke() and bench.py's CPU legs.
 *
 * Reference files cited below are relative to the reference project root;
 * "cnic/" abbreviates TAC_training_backend/spmm_cnic/.
 */
#include "tcc_oracle.h"

#include <stdlib.h>
#include <string.h>
#include <stdio.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------ utilities --- */

static int popc8(uint32_t v) { return __builtin_popcount(v & 0xFFu); }
static int popc64(uint64_t v) { return __builtin_popcountll(v); }

float orc_tf32_rna(float x) {
    uint32_t u;
    memcpy(&u, &x, 4);
    if ((u & 0x7F800000u) == 0x7F800000u) return x; /* inf / nan unchanged */
    u = (u + 0x1000u) & 0xFFFFE000u;                 /* half-ulp, then truncate */
    float r;
    memcpy(&r, &u, 4);
    return r;
}

float orc_kat_feature(uint32_t source, uint32_t feature) {
    /* src/swtcf_spmm_main.cu:33-45: a(s) + b(s) * f, all uint32 / float maths */
    const uint32_t a = (source * 17u + 13u) % 97u;
    const uint32_t b = (source * 29u + 7u) % 89u;
    const float fa = (float)a * 0.001f;
    const float fb = (float)b * 0.00001f;
    return fa + fb * (float)feature;
}

/* LSD radix sort of n 64-bit keys, 11-bit digits; passes whose digit is constant
 * over all keys are skipped.  Result in `a`. */
static int radix_sort_u64(uint64_t* a, size_t n) {
    if (n < 2) return 0;
    uint64_t* tmp = (uint64_t*)malloc(n * sizeof(uint64_t));
    size_t* hist = (size_t*)malloc(2048 * sizeof(size_t));
    if (!tmp || !hist) { free(tmp); free(hist); return -1; }
    uint64_t* src = a;
    uint64_t* dstb = tmp;
    for (int shift = 0; shift < 64; shift += 11) {
        memset(hist, 0, 2048 * sizeof(size_t));
        for (size_t i = 0; i < n; ++i) hist[(src[i] >> shift) & 2047u]++;
        int single = 0;
        for (int d = 0; d < 2048; ++d) if (hist[d] == n) { single = 1; break; }
        if (single) continue;
        size_t run = 0;
        for (int d = 0; d < 2048; ++d) { size_t c = hist[d]; hist[d] = run; run += c; }
        for (size_t i = 0; i < n; ++i) dstb[hist[(src[i] >> shift) & 2047u]++] = src[i];
        uint64_t* t = src; src = dstb; dstb = t;
    }
    if (src != a) memcpy(a, src, n * sizeof(uint64_t));
    free(tmp);
    free(hist);
    return 0;
}

/* Window groups shared by SWTCF, BCSR and BCSC: every pair (x, y) falls into
 * window x>>3 with local bit x&7; a group is one distinct (window, y) with the
 * OR of its local bits.  Groups come out sorted by (window, y)
 * (src/swtcf_convert.cu:104-144 keys, :1951-1990 sort + run-length encode). */
typedef struct {
    size_t n;          /* number of groups */
    uint32_t* win;     /* window of each group */
    uint32_t* y;       /* group key within the window */
    uint8_t* mask;     /* OR of local bits */
    uint64_t* start;   /* first group of each window, nwin+1 entries */
} groups_t;

static void groups_free(groups_t* g) {
    free(g->win); free(g->y); free(g->mask); free(g->start);
    memset(g, 0, sizeof(*g));
}

static int build_groups(size_t npairs, const uint32_t* xs, const uint32_t* ys,
                        uint32_t nwin, groups_t* out) {
    memset(out, 0, sizeof(*out));
    uint64_t* keys = (uint64_t*)malloc((npairs ? npairs : 1) * sizeof(uint64_t));
    if (!keys) return ORC_ERR_ARG;
    for (size_t e = 0; e < npairs; ++e) {
        keys[e] = ((uint64_t)(xs[e] >> 3) << 35) | ((uint64_t)ys[e] << 3) | (uint64_t)(xs[e] & 7u);
    }
    if (radix_sort_u64(keys, npairs) != 0) { free(keys); return ORC_ERR_ARG; }
    size_t ng = 0;
    for (size_t e = 0; e < npairs; ++e) {
        if (e == 0 || (keys[e] >> 3) != (keys[e - 1] >> 3)) ++ng;
    }
    out->win = (uint32_t*)malloc((ng ? ng : 1) * sizeof(uint32_t));
    out->y = (uint32_t*)malloc((ng ? ng : 1) * sizeof(uint32_t));
    out->mask = (uint8_t*)calloc(ng ? ng : 1, 1);
    out->start = (uint64_t*)calloc((size_t)nwin + 1, sizeof(uint64_t));
    if (!out->win || !out->y || !out->mask || !out->start) { free(keys); groups_free(out); return ORC_ERR_ARG; }
    size_t g = (size_t)-1;
    for (size_t e = 0; e < npairs; ++e) {
        if (e == 0 || (keys[e] >> 3) != (keys[e - 1] >> 3)) {
            ++g;
            out->win[g] = (uint32_t)(keys[e] >> 35);
            out->y[g] = (uint32_t)((keys[e] >> 3) & 0xFFFFFFFFu);
            out->mask[g] = 0;
        }
        const uint8_t bit = (uint8_t)(1u << (keys[e] & 7u));
        if (out->mask[g] & bit) { free(keys); groups_free(out); return ORC_ERR_DUPLICATE; }
        out->mask[g] |= bit;
    }
    out->n = ng;
    for (size_t i = 0; i < ng; ++i) out->start[out->win[i] + 1]++;
    for (uint32_t w = 0; w < nwin; ++w) out->start[w + 1] += out->start[w];
    free(keys);
    return ORC_OK;
}

/* ---------------------------------------------------------------- SWTCF --- */

int orc_swtcf_convert(uint32_t rows, uint32_t cols, uint32_t S, uint64_t nnz,
                      const uint32_t* dst, const uint32_t* src, uint64_t cap_tiles,
                      uint64_t cap_rows, uint32_t* colWindowOffset, uint64_t* tileLocalBit,
                      uint32_t* tileRowSlot, uint32_t* superWindowRowOffset,
                      uint32_t* superWindowRows, uint8_t* superWindowRowCacheSlot,
                      uint32_t* superWindowCachedRowSlot, uint8_t* superWindowCachedCount,
                      uint64_t* num_tiles, uint64_t* num_rows) {
    /* argument rules of src/swtcf_convert.cu:1120-1130 and :1762-1777 */
    if (cols == 0 || nnz == 0 || S == 0 || S > 32) return ORC_ERR_ARG;
    for (uint64_t e = 0; e < nnz; ++e) {
        if (dst[e] >= rows || src[e] >= cols) return ORC_ERR_RANGE;
    }
    const uint32_t W = (cols + ORC_WINDOW - 1) / ORC_WINDOW;     /* :1150-1156 */
    const uint32_t SW = (W + S - 1) / S;                         /* :1158-1164 */
    groups_t g;
    int st = build_groups((size_t)nnz, src, dst, W, &g);
    if (st != ORC_OK) return st;

    /* degree-descending order inside each window (:216-265, :292-376), ties by dst */
    uint64_t* pos = (uint64_t*)malloc((g.n ? g.n : 1) * sizeof(uint64_t));
    colWindowOffset[0] = 0;
    uint64_t T = 0;
    for (uint32_t w = 0; w < W; ++w) {
        uint64_t p = 0;
        for (int d = 8; d >= 1; --d) {
            for (uint64_t i = g.start[w]; i < g.start[w + 1]; ++i) {
                if (popc8(g.mask[i]) == d) pos[i] = p++;
            }
        }
        T += (p + 7) / 8;
        if (T > 0xFFFFFFFFull) { free(pos); groups_free(&g); return ORC_ERR_CAPACITY; }
        colWindowOffset[w + 1] = (uint32_t)T;
    }
    if (T > cap_tiles) { free(pos); groups_free(&g); return ORC_ERR_CAPACITY; }

    /* unique (superWindow, dst) rows ascending with window occurrence (:459-681) */
    uint64_t* swkeys = (uint64_t*)malloc((g.n ? g.n : 1) * sizeof(uint64_t));
    for (size_t i = 0; i < g.n; ++i) swkeys[i] = ((uint64_t)(g.win[i] / S) << 32) | g.y[i];
    radix_sort_u64(swkeys, g.n);
    uint64_t R = 0;
    memset(superWindowRowOffset, 0, ((size_t)SW + 1) * sizeof(uint32_t));
    uint32_t* occ = (uint32_t*)malloc((g.n ? g.n : 1) * sizeof(uint32_t));
    for (size_t i = 0; i < g.n; ++i) {
        if (i == 0 || swkeys[i] != swkeys[i - 1]) {
            if (R >= cap_rows) { free(occ); free(swkeys); free(pos); groups_free(&g); return ORC_ERR_CAPACITY; }
            superWindowRows[R] = (uint32_t)(swkeys[i] & 0xFFFFFFFFu);
            occ[R] = 0;
            superWindowRowOffset[(swkeys[i] >> 32) + 1]++;
            ++R;
        }
        occ[R - 1]++;
    }
    for (uint32_t s = 0; s < SW; ++s) superWindowRowOffset[s + 1] += superWindowRowOffset[s];

    /* tiles: bitmaps (:379-456) and row slots (:898-1107) */
    for (uint64_t t = 0; t < T; ++t) tileLocalBit[t] = 0;
    for (uint64_t i = 0; i < 8 * T; ++i) tileRowSlot[i] = ORC_INVALID_SLOT;
    for (size_t i = 0; i < g.n; ++i) {
        const uint32_t w = g.win[i];
        const uint32_t s = w / S;
        const uint64_t tile = colWindowOffset[w] + pos[i] / 8;
        const uint32_t lr = (uint32_t)(pos[i] % 8);
        tileLocalBit[tile] |= (uint64_t)g.mask[i] << (8 * lr);
        /* slot = rank of dst among the super-window's ascending rows */
        uint64_t lo = superWindowRowOffset[s], hi = superWindowRowOffset[s + 1];
        while (lo < hi) {
            uint64_t mid = (lo + hi) / 2;
            if (superWindowRows[mid] < g.y[i]) lo = mid + 1; else hi = mid;
        }
        tileRowSlot[tile * 8 + lr] = (uint32_t)(lo - superWindowRowOffset[s]);
    }

    /* repeat cache (:699-895): rows seen in >= 2 windows, occurrence descending,
     * slot ascending; the first 32 get cache slots */
    memset(superWindowRowCacheSlot, 0xFF, (size_t)R);
    memset(superWindowCachedRowSlot, 0xFF, (size_t)SW * ORC_CACHE * sizeof(uint32_t));
    for (uint32_t s = 0; s < SW; ++s) {
        const uint32_t b = superWindowRowOffset[s], e = superWindowRowOffset[s + 1];
        uint32_t rank = 0;
        for (int o = (int)S; o >= 2 && rank < ORC_CACHE; --o) {
            for (uint32_t r = b; r < e && rank < ORC_CACHE; ++r) {
                if (occ[r] == (uint32_t)o) {
                    superWindowRowCacheSlot[r] = (uint8_t)rank;
                    superWindowCachedRowSlot[(size_t)s * ORC_CACHE + rank] = r - b;
                    ++rank;
                }
            }
        }
        superWindowCachedCount[s] = (uint8_t)rank;
    }
    *num_tiles = T;
    *num_rows = R;
    free(occ); free(swkeys); free(pos);
    groups_free(&g);
    return ORC_OK;
}

static void set_why(char* why, size_t len, const char* msg) {
    if (why && len) { strncpy(why, msg, len - 1); why[len - 1] = 0; }
}

static int cmp_u64(const void* a, const void* b) {
    const uint64_t x = *(const uint64_t*)a, y = *(const uint64_t*)b;
    return x < y ? -1 : x > y;
}

int orc_swtcf_validate(uint32_t cols, uint32_t S, uint64_t nnz, const uint32_t* dst,
                       const uint32_t* src, uint32_t W, const uint32_t* colWindowOffset,
                       const uint64_t* tileLocalBit, const uint32_t* tileRowSlot, uint32_t SW,
                       const uint32_t* superWindowRowOffset, const uint32_t* superWindowRows,
                       const uint8_t* superWindowRowCacheSlot,
                       const uint32_t* superWindowCachedRowSlot,
                       const uint8_t* superWindowCachedCount, char* why, size_t why_len) {
    /* validateSWTCF, src/swtcf_convert_main.cu:36-130 */
    uint64_t* expect = (uint64_t*)malloc((nnz ? nnz : 1) * 8);
    uint64_t* got = (uint64_t*)malloc((nnz ? nnz : 1) * 8);
    uint64_t ng = 0;
    int ok = 1;
    for (uint64_t e = 0; e < nnz; ++e) expect[e] = ((uint64_t)dst[e] << 32) | src[e];
    for (uint32_t w = 0; w < W && ok; ++w) {
        const uint32_t s = w / S;
        const uint32_t sb = superWindowRowOffset[s], se = superWindowRowOffset[s + 1];
        int prev = 9;
        for (uint32_t t = colWindowOffset[w]; t < colWindowOffset[w + 1] && ok; ++t) {
            for (uint32_t lr = 0; lr < 8 && ok; ++lr) {
                const uint32_t bits = (uint32_t)((tileLocalBit[t] >> (8 * lr)) & 0xFFu);
                const uint32_t slot = tileRowSlot[(size_t)t * 8 + lr];
                if (bits == 0) {
                    if (slot != ORC_INVALID_SLOT) { set_why(why, why_len, "padding slot is not INVALID"); ok = 0; }
                    continue;
                }
                const int d = popc8(bits);
                if (d > prev) { set_why(why, why_len, "row reorder is not degree descending"); ok = 0; break; }
                prev = d;
                if (slot >= se - sb) { set_why(why, why_len, "invalid row slot"); ok = 0; break; }
                const uint32_t gd = superWindowRows[sb + slot];
                for (uint32_t k = 0; k < 8; ++k) {
                    if (!(bits & (1u << k))) continue;
                    const uint32_t gs = w * 8 + k;
                    if (gs >= cols) { set_why(why, why_len, "src exceeds numSrc"); ok = 0; break; }
                    if (ng >= nnz) { set_why(why, why_len, "edge count mismatch"); ok = 0; break; }
                    got[ng++] = ((uint64_t)gd << 32) | gs;
                }
            }
        }
    }
    if (ok) {
        qsort(expect, (size_t)nnz, 8, cmp_u64);
        qsort(got, (size_t)ng, 8, cmp_u64);
        if (ng != nnz) { set_why(why, why_len, "edge count mismatch"); ok = 0; }
        else if (memcmp(expect, got, (size_t)nnz * 8) != 0) { set_why(why, why_len, "COO reconstruction mismatch"); ok = 0; }
    }
    free(expect); free(got);
    if (!ok) return ORC_ERR_VALIDATE;

    /* validateRepeatCacheMetadata, src/swtcf_convert_main.cu:132-310 */
    for (uint32_t s = 0; s < SW && ok; ++s) {
        const uint32_t rb = superWindowRowOffset[s], re = superWindowRowOffset[s + 1];
        const uint32_t rc = re - rb;
        uint32_t* occ = (uint32_t*)calloc(rc ? rc : 1, 4);
        uint8_t* cached = (uint8_t*)calloc(rc ? rc : 1, 1);
        const uint32_t wb = s * S, we = (wb + S < W) ? wb + S : W;
        for (uint32_t w = wb; w < we && ok; ++w)
            for (uint32_t t = colWindowOffset[w]; t < colWindowOffset[w + 1] && ok; ++t)
                for (uint32_t lr = 0; lr < 8; ++lr) {
                    if (((tileLocalBit[t] >> (8 * lr)) & 0xFFu) == 0) continue;
                    const uint32_t slot = tileRowSlot[(size_t)t * 8 + lr];
                    if (slot >= rc) { set_why(why, why_len, "cache validation: rowSlot out of range"); ok = 0; break; }
                    occ[slot]++;
                }
        uint32_t repeated = 0;
        for (uint32_t r = 0; r < rc && ok; ++r) {
            if (occ[r] == 0) { set_why(why, why_len, "cache validation: unused row"); ok = 0; }
            if (occ[r] > 1) ++repeated;
        }
        const uint32_t expect_cached = repeated < ORC_CACHE ? repeated : ORC_CACHE;
        const uint32_t cc = superWindowCachedCount[s];
        if (ok && cc != expect_cached) { set_why(why, why_len, "cache validation: cachedCount mismatch"); ok = 0; }
        uint32_t min_cached = 0xFFFFFFFFu, max_uncached = 0;
        uint8_t seen[ORC_CACHE];
        memset(seen, 0, sizeof(seen));
        for (uint32_t c = 0; c < ORC_CACHE && ok; ++c) {
            const uint32_t slot = superWindowCachedRowSlot[(size_t)s * ORC_CACHE + c];
            if (c < cc) {
                if (slot >= rc) { set_why(why, why_len, "cache validation: cached rowSlot invalid"); ok = 0; break; }
                if (occ[slot] <= 1) { set_why(why, why_len, "cache validation: non-repeated row cached"); ok = 0; break; }
                if (cached[slot]) { set_why(why, why_len, "cache validation: row cached twice"); ok = 0; break; }
                if (seen[c]) { set_why(why, why_len, "cache validation: cache slot duplicated"); ok = 0; break; }
                cached[slot] = 1;
                seen[c] = 1;
                if (superWindowRowCacheSlot[rb + slot] != (uint8_t)c) { set_why(why, why_len, "cache validation: forward/reverse mismatch"); ok = 0; break; }
                if (occ[slot] < min_cached) min_cached = occ[slot];
            } else if (slot != ORC_INVALID_SLOT) {
                set_why(why, why_len, "cache validation: unused cache entry is not INVALID"); ok = 0; break;
            }
        }
        for (uint32_t r = 0; r < rc && ok; ++r) {
            const uint8_t cs = superWindowRowCacheSlot[rb + r];
            if (cached[r]) {
                if (cs >= ORC_CACHE) { set_why(why, why_len, "cache validation: cached row has invalid slot"); ok = 0; }
            } else {
                if (cs != ORC_INVALID_CACHE) { set_why(why, why_len, "cache validation: uncached row has slot"); ok = 0; }
                if (occ[r] > 1 && occ[r] > max_uncached) max_uncached = occ[r];
            }
        }
        if (ok && repeated > ORC_CACHE && min_cached < max_uncached) {
            set_why(why, why_len, "cache validation: top-H priority violated"); ok = 0;
        }
        free(occ); free(cached);
    }
    return ok ? ORC_OK : ORC_ERR_VALIDATE;
}

typedef struct { uint32_t dst; uint8_t mask; uint8_t deg; } orow_t;

static int cmp_orow(const void* a, const void* b) {
    const orow_t* x = (const orow_t*)a;
    const orow_t* y = (const orow_t*)b;
    if (x->deg != y->deg) return x->deg > y->deg ? -1 : 1;
    return x->dst < y->dst ? -1 : x->dst > y->dst;
}

static int cmp_u32(const void* a, const void* b) {
    const uint32_t x = *(const uint32_t*)a, y = *(const uint32_t*)b;
    return x < y ? -1 : x > y;
}

int orc_swtcf_canonicalize(uint32_t S, uint32_t W, const uint32_t* colWindowOffset,
                           uint64_t* tileLocalBit, uint32_t* tileRowSlot, uint32_t SW,
                           const uint32_t* superWindowRowOffset, uint32_t* superWindowRows,
                           uint8_t* superWindowRowCacheSlot, uint32_t* superWindowCachedRowSlot,
                           uint8_t* superWindowCachedCount) {
    for (uint32_t s = 0; s < SW; ++s) {
        const uint32_t rb = superWindowRowOffset[s], re = superWindowRowOffset[s + 1];
        const uint32_t rc = re - rb;
        /* 1. super-window rows ascending; old slot -> new slot */
        uint32_t* sorted = (uint32_t*)malloc((rc ? rc : 1) * 4);
        memcpy(sorted, superWindowRows + rb, (size_t)rc * 4);
        qsort(sorted, rc, 4, cmp_u32);
        uint32_t* newslot = (uint32_t*)malloc((rc ? rc : 1) * 4);
        for (uint32_t r = 0; r < rc; ++r) {
            const uint32_t d = superWindowRows[rb + r];
            uint32_t lo = 0, hi = rc;
            while (lo < hi) { uint32_t mid = (lo + hi) / 2; if (sorted[mid] < d) lo = mid + 1; else hi = mid; }
            if (lo >= rc || sorted[lo] != d) { free(sorted); free(newslot); return ORC_ERR_VALIDATE; }
            newslot[r] = lo;
        }
        uint32_t* occ = (uint32_t*)calloc(rc ? rc : 1, 4);
        /* 2. each window: rows by degree descending then dst ascending */
        const uint32_t wb = s * S, we = (wb + S < W) ? wb + S : W;
        for (uint32_t w = wb; w < we; ++w) {
            const uint32_t tb = colWindowOffset[w], te = colWindowOffset[w + 1];
            const size_t cap = (size_t)(te - tb) * 8;
            orow_t* rowsv = (orow_t*)malloc((cap ? cap : 1) * sizeof(orow_t));
            size_t n = 0;
            for (uint32_t t = tb; t < te; ++t)
                for (uint32_t lr = 0; lr < 8; ++lr) {
                    const uint32_t bits = (uint32_t)((tileLocalBit[t] >> (8 * lr)) & 0xFFu);
                    if (!bits) continue;
                    const uint32_t slot = tileRowSlot[(size_t)t * 8 + lr];
                    if (slot >= rc) { free(rowsv); free(occ); free(sorted); free(newslot); return ORC_ERR_VALIDATE; }
                    rowsv[n].dst = superWindowRows[rb + slot];
                    rowsv[n].mask = (uint8_t)bits;
                    rowsv[n].deg = (uint8_t)popc8(bits);
                    ++n;
                }
            qsort(rowsv, n, sizeof(orow_t), cmp_orow);
            for (uint32_t t = tb; t < te; ++t) tileLocalBit[t] = 0;
            for (size_t i = 0; i < cap; ++i) tileRowSlot[(size_t)tb * 8 + i] = ORC_INVALID_SLOT;
            for (size_t p = 0; p < n; ++p) {
                const uint32_t t = tb + (uint32_t)(p / 8), lr = (uint32_t)(p % 8);
                tileLocalBit[t] |= (uint64_t)rowsv[p].mask << (8 * lr);
                uint32_t lo = 0, hi = rc;
                while (lo < hi) { uint32_t mid = (lo + hi) / 2; if (sorted[mid] < rowsv[p].dst) lo = mid + 1; else hi = mid; }
                tileRowSlot[(size_t)t * 8 + lr] = lo;
                occ[lo]++;
            }
            free(rowsv);
        }
        memcpy(superWindowRows + rb, sorted, (size_t)rc * 4);
        /* 3. cache ranks: occurrence descending, slot ascending */
        memset(superWindowRowCacheSlot + rb, 0xFF, rc);
        for (uint32_t c = 0; c < ORC_CACHE; ++c) superWindowCachedRowSlot[(size_t)s * ORC_CACHE + c] = ORC_INVALID_SLOT;
        uint32_t rank = 0;
        for (int o = (int)S; o >= 2 && rank < ORC_CACHE; --o)
            for (uint32_t r = 0; r < rc && rank < ORC_CACHE; ++r)
                if (occ[r] == (uint32_t)o) {
                    superWindowRowCacheSlot[rb + r] = (uint8_t)rank;
                    superWindowCachedRowSlot[(size_t)s * ORC_CACHE + rank] = r;
                    ++rank;
                }
        superWindowCachedCount[s] = (uint8_t)rank;
        free(occ); free(sorted); free(newslot);
    }
    return ORC_OK;
}

void orc_swtcf_spmm(uint32_t W, uint32_t S, uint32_t cols, const uint32_t* colWindowOffset,
                    const uint64_t* tileLocalBit, const uint32_t* tileRowSlot,
                    const uint32_t* superWindowRowOffset, const uint32_t* superWindowRows,
                    const float* X, uint32_t F, uint64_t ldx, float* Y, uint64_t ldy,
                    uint32_t thr) {
    /* src/swtcf_spmm.cu:105-265: per tile row, sum the window's X rows selected
     * by the row's 8 bits; dense tiles go through TF32 (A = X rounded rna). */
    for (uint32_t w = 0; w < W; ++w) {
        const uint32_t s = w / S;
        const uint32_t rb = superWindowRowOffset[s];
        for (uint32_t t = colWindowOffset[w]; t < colWindowOffset[w + 1]; ++t) {
            const uint64_t bm = tileLocalBit[t];
            const int tc = (uint32_t)popc64(bm) >= thr;
            for (uint32_t lr = 0; lr < 8; ++lr) {
                const uint32_t bits = (uint32_t)((bm >> (8 * lr)) & 0xFFu);
                const uint32_t slot = tileRowSlot[(size_t)t * 8 + lr];
                if (!bits || slot == ORC_INVALID_SLOT) continue;
                const uint32_t row = superWindowRows[rb + slot];
                for (uint32_t f = 0; f < F; ++f) {
                    float acc = 0.f;
                    for (uint32_t k = 0; k < 8; ++k) {
                        if (!(bits & (1u << k))) continue;
                        const uint32_t c = w * 8 + k;
                        if (c >= cols) continue;
                        const float v = X[(size_t)c * ldx + f];
                        acc += tc ? orc_tf32_rna(v) : v;
                    }
                    Y[(size_t)row * ldy + f] += acc;
                }
            }
        }
    }
}

/* ------------------------------------------------------------ BCSR/BCSC --- */

static int tiles_from_groups(const groups_t* g, uint32_t nwin, int bit_is_row_major,
                             uint64_t cap_tiles, uint32_t* winOffset, uint32_t* tcOffset,
                             uint32_t* idx, uint64_t* bits, uint64_t* num_tiles) {
    /* Tile t of window w holds the window's groups 8(t-off[w]) .. +7; group k of
     * the tile contributes its mask at bit i*8+k (BCSR, mask bit i = local row)
     * or at bit k*8+n... expressed for BCSC as (position n)*8 + (local col bit). */
    uint64_t T = 0;
    if (winOffset) winOffset[0] = 0;
    for (uint32_t w = 0; w < nwin; ++w) {
        const uint64_t n = g->start[w + 1] - g->start[w];
        T += (n + 7) / 8;
        if (T > 0xFFFFFFFFull) return ORC_ERR_CAPACITY;
        if (winOffset) winOffset[w + 1] = (uint32_t)T;
    }
    *num_tiles = T;
    if (!idx) return ORC_OK;
    if (T > cap_tiles) return ORC_ERR_CAPACITY;
    for (uint64_t i = 0; i < 8 * T; ++i) idx[i] = ORC_INVALID_SLOT;
    for (uint64_t t = 0; t < T; ++t) bits[t] = 0;
    for (uint32_t w = 0; w < nwin; ++w) {
        const uint64_t tb = winOffset[w];
        for (uint64_t i = g->start[w]; i < g->start[w + 1]; ++i) {
            const uint64_t p = i - g->start[w];
            const uint64_t t = tb + p / 8;
            const uint32_t k = (uint32_t)(p % 8);
            idx[t * 8 + k] = g->y[i];
            const uint32_t m = g->mask[i];
            if (bit_is_row_major) {
                for (uint32_t r = 0; r < 8; ++r)
                    if (m & (1u << r)) bits[t] |= 1ull << (r * 8 + k);
            } else {
                bits[t] |= (uint64_t)m << (8 * k);
            }
        }
    }
    if (tcOffset) {
        tcOffset[0] = 0;
        for (uint64_t t = 0; t < T; ++t) tcOffset[t + 1] = tcOffset[t] + (uint32_t)popc64(bits[t]);
    }
    return ORC_OK;
}

static int csr_pairs(uint32_t rows, uint32_t cols, const uint64_t* rowptr, const uint32_t* col,
                     uint32_t** rs, uint32_t** cs) {
    const uint64_t nnz = rowptr[rows];
    *rs = (uint32_t*)malloc((nnz ? nnz : 1) * 4);
    *cs = (uint32_t*)malloc((nnz ? nnz : 1) * 4);
    if (!*rs || !*cs) return ORC_ERR_ARG;
    for (uint32_t r = 0; r < rows; ++r) {
        if (rowptr[r + 1] < rowptr[r]) return ORC_ERR_ARG;
        for (uint64_t j = rowptr[r]; j < rowptr[r + 1]; ++j) {
            if (col[j] >= cols) return ORC_ERR_RANGE;
            (*rs)[j] = r;
            (*cs)[j] = col[j];
        }
    }
    return ORC_OK;
}

int orc_bcsr_from_csr(uint32_t rows, uint32_t cols, const uint64_t* rowptr, const uint32_t* col,
                      uint64_t cap_tiles, uint32_t* rowWindowOffset, uint32_t* tcOffset,
                      uint32_t* sparseA2B, uint64_t* tcLocalBit, uint64_t* num_tiles) {
    uint32_t *rs = NULL, *cs = NULL;
    int st = csr_pairs(rows, cols, rowptr, col, &rs, &cs);
    if (st != ORC_OK) { free(rs); free(cs); return st; }
    const uint32_t nwin = (rows + 7) / 8;
    groups_t g;
    /* window = row>>3, group key = column, local bit = row&7 */
    st = build_groups((size_t)rowptr[rows], rs, cs, nwin, &g);
    free(rs); free(cs);
    if (st != ORC_OK) return st;
    st = tiles_from_groups(&g, nwin, 1, cap_tiles, rowWindowOffset, tcOffset, sparseA2B, tcLocalBit, num_tiles);
    groups_free(&g);
    return st;
}

int orc_bcsc_from_csr(uint32_t rows, uint32_t cols, const uint64_t* rowptr, const uint32_t* col,
                      uint64_t cap_tiles, uint32_t* colWindowOffset, uint32_t* tcOffset,
                      uint32_t* sparseA2C, uint64_t* tcLocalBit, uint64_t* num_tiles) {
    uint32_t *rs = NULL, *cs = NULL;
    int st = csr_pairs(rows, cols, rowptr, col, &rs, &cs);
    if (st != ORC_OK) { free(rs); free(cs); return st; }
    const uint32_t nwin = (cols + 7) / 8;
    groups_t g;
    /* window = col>>3, group key = row, local bit = col&7 */
    st = build_groups((size_t)rowptr[rows], cs, rs, nwin, &g);
    free(rs); free(cs);
    if (st != ORC_OK) return st;
    st = tiles_from_groups(&g, nwin, 0, cap_tiles, colWindowOffset, tcOffset, sparseA2C, tcLocalBit, num_tiles);
    groups_free(&g);
    return st;
}

void orc_bcsr_spmm(uint32_t nwin, uint32_t num_cols, const uint32_t* rowWindowOffset,
                   const uint32_t* sparseA2B, const uint64_t* tcLocalBit, const float* B,
                   uint32_t F, uint64_t ldb, float* C, uint64_t ldc, uint32_t num_rows,
                   uint32_t thr) {
    /* cnic/src/core/spmm_kernel.cu:1560-1843: C[8w+i] += sum_k bit(i*8+k) B[A2B[k]] */
    for (uint32_t w = 0; w < nwin; ++w)
        for (uint32_t t = rowWindowOffset[w]; t < rowWindowOffset[w + 1]; ++t) {
            const uint64_t bm = tcLocalBit[t];
            const int tc = (uint32_t)popc64(bm) >= thr;
            for (uint32_t i = 0; i < 8; ++i) {
                const uint32_t row = w * 8 + i;
                if (row >= num_rows || !((bm >> (8 * i)) & 0xFFu)) continue;
                for (uint32_t f = 0; f < F; ++f) {
                    float acc = 0.f;
                    for (uint32_t k = 0; k < 8; ++k) {
                        if (!((bm >> (8 * i + k)) & 1u)) continue;
                        const uint32_t c = sparseA2B[(size_t)t * 8 + k];
                        if (c >= num_cols) continue;
                        const float v = B[(size_t)c * ldb + f];
                        acc += tc ? orc_tf32_rna(v) : v;
                    }
                    C[(size_t)row * ldc + f] += acc;
                }
            }
        }
}

void orc_bcsc_spmm(uint32_t nwin, uint32_t num_cols, const uint32_t* colWindowOffset,
                   const uint32_t* sparseA2C, const uint64_t* tcLocalBit, const float* B,
                   uint32_t F, uint64_t ldb, float* C, uint64_t ldc, uint32_t num_rows,
                   uint32_t thr) {
    /* cnic/src/core/spmm_kernel.cu:1844-2167: B rows 8c..8c+7 pushed into
     * C[A2C[n]] (guard A2C[n] < numRows, :2067/:2078) */
    for (uint32_t w = 0; w < nwin; ++w)
        for (uint32_t t = colWindowOffset[w]; t < colWindowOffset[w + 1]; ++t) {
            const uint64_t bm = tcLocalBit[t];
            const int tc = (uint32_t)popc64(bm) >= thr;
            for (uint32_t n = 0; n < 8; ++n) {
                const uint32_t row = sparseA2C[(size_t)t * 8 + n];
                const uint32_t bits = (uint32_t)((bm >> (8 * n)) & 0xFFu);
                if (row >= num_rows || !bits) continue;
                for (uint32_t f = 0; f < F; ++f) {
                    float acc = 0.f;
                    for (uint32_t k = 0; k < 8; ++k) {
                        if (!(bits & (1u << k))) continue;
                        const uint32_t c = w * 8 + k;
                        if (c >= num_cols) continue;
                        const float v = B[(size_t)c * ldb + f];
                        acc += tc ? orc_tf32_rna(v) : v;
                    }
                    C[(size_t)row * ldc + f] += acc;
                }
            }
        }
}

/* ------------------------------------------------------------- CSR SpMM --- */

void orc_csr_spmm(uint32_t rows, const uint64_t* rowptr, const uint32_t* col, const float* rs,
                  const float* cs, const float* X, uint32_t F, uint64_t ldx, float* Y,
                  uint64_t ldy, int accumulate) {
    double* acc = (double*)malloc((F ? F : 1) * sizeof(double));
    for (uint32_t r = 0; r < rows; ++r) {
        for (uint32_t f = 0; f < F; ++f) acc[f] = 0.0;
        for (uint64_t j = rowptr[r]; j < rowptr[r + 1]; ++j) {
            const uint32_t c = col[j];
            const double w = cs ? (double)cs[c] : 1.0;
            const float* x = X + (size_t)c * ldx;
            for (uint32_t f = 0; f < F; ++f) acc[f] += w * (double)x[f];
        }
        const double s = rs ? (double)rs[r] : 1.0;
        float* y = Y + (size_t)r * ldy;
        for (uint32_t f = 0; f < F; ++f) {
            const float v = (float)(s * acc[f]);
            y[f] = accumulate ? y[f] + v : v;
        }
    }
    free(acc);
}

void orc_csr_spmm_t(uint32_t rows, uint32_t cols, const uint64_t* rowptr, const uint32_t* col,
                    const float* rs, const float* cs, const float* X, uint32_t F, uint64_t ldx,
                    float* Y, uint64_t ldy, int accumulate) {
    double* acc = (double*)calloc((size_t)cols * F + 1, sizeof(double));
    for (uint32_t r = 0; r < rows; ++r) {
        const double s = rs ? (double)rs[r] : 1.0;
        const float* x = X + (size_t)r * ldx;
        for (uint64_t j = rowptr[r]; j < rowptr[r + 1]; ++j) {
            double* a = acc + (size_t)col[j] * F;
            for (uint32_t f = 0; f < F; ++f) a[f] += s * (double)x[f];
        }
    }
    for (uint32_t c = 0; c < cols; ++c) {
        const double w = cs ? (double)cs[c] : 1.0;
        float* y = Y + (size_t)c * ldy;
        for (uint32_t f = 0; f < F; ++f) {
            const float v = (float)(w * acc[(size_t)c * F + f]);
            y[f] = accumulate ? y[f] + v : v;
        }
    }
    free(acc);
}

void orc_csr_spmm_f32_omp(uint32_t rows, const uint64_t* rowptr, const uint32_t* col,
                          const float* rs, const float* cs, const float* X, uint32_t F,
                          uint64_t ldx, float* Y, uint64_t ldy, int threads) {
#ifdef _OPENMP
    if (threads > 0) omp_set_num_threads(threads);
#else
    (void)threads;
#endif
#pragma omp parallel
    {
        float* acc = (float*)malloc((F ? F : 1) * sizeof(float));
#pragma omp for schedule(dynamic, 64)
        for (long long r = 0; r < (long long)rows; ++r) {
            for (uint32_t f = 0; f < F; ++f) acc[f] = 0.f;
            for (uint64_t j = rowptr[r]; j < rowptr[r + 1]; ++j) {
                const uint32_t c = col[j];
                const float w = cs ? cs[c] : 1.f;
                const float* x = X + (size_t)c * ldx;
                for (uint32_t f = 0; f < F; ++f) acc[f] += w * x[f];
            }
            const float s = rs ? rs[r] : 1.f;
            float* y = Y + (size_t)r * ldy;
            for (uint32_t f = 0; f < F; ++f) y[f] = s * acc[f];
        }
        free(acc);
    }
}
