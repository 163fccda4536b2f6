/*
 * TEST INFRASTRUCTURE — the CPU oracle for the radix codec's hot path.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg may
 * load this library, and only as the checker. Nothing in drinkme_b200/ links
 * or calls it; the product path is CUDA and fails loudly without its
 * extension.
 *
 * A plain-C restatement of the reference's CPU algorithm for BF16 radix
 * tensors (pack format 1), written from its published behaviour:
 *
 *   block_word_bounds   src/drinkme/codec/radix.py:149-171
 *   validate            src/drinkme/codec/radix.py:174-238
 *   decode              src/drinkme/codec/radix.py:241-278
 *                       (same bits as radix_native.cpp:168-209)
 *   schedule            src/drinkme/codec/radix_pack.py:353-411 (schedule_np)
 *   linear (float64)    the oracle of bench/radix_gemv_bitpin.py:181-186:
 *                       y = x @ W^T in float64 and |x| @ |W|^T for the bound
 *
 * Stream layout (docs/pack-format.md, "radix"): per block of n weights,
 * whole-word streams in order: n 8-bit literals (sign << 7 | mantissa),
 * then for every nonterminal tier k a w_k-bit code per weight still active
 * (code 2^w_k - 1 escapes to the next tier), then an 8-bit exponent per
 * weight that escaped every tier. Fields are little-endian inside uint32
 * words; a field may straddle two words.
 */
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#define MANT 7
#define EXPB 8

static void set_err(char *err, size_t len, const char *msg) {
    if (err && len) {
        strncpy(err, msg, len - 1);
        err[len - 1] = 0;
    }
}

/* Field `index` of a `width`-bit little-endian stream starting at word 0 of
 * `words` (the caller guarantees the words it touches exist). */
static uint32_t field(const uint32_t *words, uint64_t index, uint32_t width) {
    uint64_t bit = index * width;
    uint32_t lo = (uint32_t)(bit & 31);
    uint64_t v = words[bit >> 5] >> lo;
    if (lo + width > 32) v |= (uint64_t)words[(bit >> 5) + 1] << (32 - lo);
    return (uint32_t)(v & ((1u << width) - 1));
}

static int64_t ceil_words(int64_t count, int64_t width) { return (count * width + 31) / 32; }

/* radix.py:149-171 — the fewest / most words a block of n weights can take. */
int oracle_word_bounds(int64_t n, const int32_t *widths, int32_t nw, int64_t *fewest, int64_t *most) {
    int64_t fixed = ceil_words(n, MANT + 1) + ceil_words(n, widths[0]);
    int64_t m = fixed;
    for (int i = 1; i < nw - 1; ++i) m += ceil_words(n, widths[i]);
    m += ceil_words(n, EXPB);
    *fewest = fixed;
    *most = m;
    return 0;
}

static int check_widths(const int32_t *widths, int32_t nw, int32_t *covered) {
    if (nw < 2 || nw > 8 || widths[nw - 1] != EXPB) return 1;
    int32_t c = 0;
    for (int i = 0; i < nw; ++i)
        if (widths[i] < 1 || widths[i] > 8) return 1;
    for (int i = 0; i < nw - 1; ++i) c += (1 << widths[i]) - 1;
    if (c > (1 << EXPB)) return 1;
    *covered = c;
    return 0;
}

/* radix.py:174-238, the descriptor checks (no payload word is read). */
int oracle_validate(int64_t R, int64_t C, int64_t B, const int32_t *widths, int32_t nw,
                    const uint8_t *palette, int64_t npal, const uint32_t *offsets, int64_t noff,
                    int64_t nwords, char *err, size_t errlen) {
    char msg[256];
    if (R <= 0 || C <= 0) { set_err(err, errlen, "invalid radix shape or raw flag"); return 1; }
    if (B < 32 || B > 4096 || (B & (B - 1))) { set_err(err, errlen, "invalid radix block size"); return 1; }
    int32_t covered;
    if (check_widths(widths, nw, &covered)) {
        set_err(err, errlen, "radix needs 2..8 widths in 1..8, ending with the exponent width");
        return 1;
    }
    int64_t per_row = (C + B - 1) / B, nb = R * per_row;
    if (npal != covered) { set_err(err, errlen, "invalid radix palette entries"); return 1; }
    {
        int seen[256] = {0};
        for (int64_t i = 0; i < npal; ++i) {
            if (seen[palette[i]]) { set_err(err, errlen, "invalid radix palette entries"); return 1; }
            seen[palette[i]] = 1;
        }
    }
    if (noff != nb + 1 || offsets[0] != 0 || (int64_t)offsets[nb] != nwords) {
        set_err(err, errlen, "invalid radix block offsets");
        return 1;
    }
    for (int64_t i = 0; i < nb; ++i)
        if (offsets[i + 1] <= offsets[i]) { set_err(err, errlen, "invalid radix block offsets"); return 1; }
    for (int64_t i = 0; i < nb; ++i) {
        int64_t n = C - (i % per_row) * B;
        if (n > B) n = B;
        int64_t length = (int64_t)offsets[i + 1] - (int64_t)offsets[i], fewest, most;
        oracle_word_bounds(n, widths, nw, &fewest, &most);
        if (length < fewest) {
            snprintf(msg, sizeof msg,
                     "invalid radix block offsets: block %lld holds %lld word(s), fewer than the %lld its "
                     "literal plane and first tier take for %lld weights",
                     (long long)i, (long long)length, (long long)fewest, (long long)n);
            set_err(err, errlen, msg);
            return 1;
        }
        if (length > most) {
            snprintf(msg, sizeof msg,
                     "invalid radix block offsets: block %lld holds %lld words, more than the %lld any block "
                     "of %lld weights can use",
                     (long long)i, (long long)length, (long long)most, (long long)n);
            set_err(err, errlen, msg);
            return 1;
        }
    }
    return 0;
}

/* radix.py:241-278 — strict decode of every block to uint16 BF16 bits. */
int oracle_decode(int64_t R, int64_t C, int64_t B, const int32_t *widths, int32_t nw,
                  const uint8_t *palette, int64_t npal, const uint32_t *offsets, int64_t noff,
                  const uint32_t *data, int64_t nwords, uint16_t *out, char *err, size_t errlen) {
    if (oracle_validate(R, C, B, widths, nw, palette, npal, offsets, noff, nwords, err, errlen)) return 1;
    int64_t per_row = (C + B - 1) / B;
    int32_t *active = (int32_t *)malloc(sizeof(int32_t) * (size_t)B);
    uint32_t *lit = (uint32_t *)malloc(sizeof(uint32_t) * (size_t)B);
    uint32_t *ex = (uint32_t *)malloc(sizeof(uint32_t) * (size_t)B);
    int rc = 0;
    for (int64_t r = 0; r < R && !rc; ++r) {
        for (int64_t b = 0; b < per_row; ++b) {
            int64_t blk = r * per_row + b;
            int64_t n = C - b * B;
            if (n > B) n = B;
            int64_t start = offsets[blk], len = (int64_t)offsets[blk + 1] - start;
            const uint32_t *s = data + start;
            int64_t pos = ceil_words(n, MANT + 1);
            if (pos > len) { set_err(err, errlen, "truncated radix stream"); rc = 1; break; }
            for (int64_t i = 0; i < n; ++i) { lit[i] = field(s, (uint64_t)i, MANT + 1); active[i] = (int32_t)i; ex[i] = 0; }
            int64_t count = n, base = 0;
            for (int t = 0; t < nw - 1; ++t) {
                uint32_t w = (uint32_t)widths[t], esc = (1u << w) - 1;
                int64_t need = ceil_words(count, w);
                if (pos + need > len) { set_err(err, errlen, "truncated radix stream"); rc = 1; break; }
                int64_t kept = 0;
                for (int64_t i = 0; i < count; ++i) {
                    uint32_t code = field(s + pos, (uint64_t)i, w);
                    if (code != esc) {
                        int64_t idx = base + code;
                        if (idx >= npal) { set_err(err, errlen, "invalid radix palette index"); rc = 1; break; }
                        ex[active[i]] = palette[idx];
                    } else {
                        active[kept++] = active[i];
                    }
                }
                if (rc) break;
                pos += need;
                count = kept;
                base += esc;
            }
            if (rc) break;
            int64_t need = ceil_words(count, EXPB);
            if (pos + need > len) { set_err(err, errlen, "truncated radix stream"); rc = 1; break; }
            for (int64_t i = 0; i < count; ++i) ex[active[i]] = field(s + pos, (uint64_t)i, EXPB);
            pos += need;
            if (pos != len) { set_err(err, errlen, "radix block has trailing words"); rc = 1; break; }
            uint16_t *dst = out + r * C + b * B;
            for (int64_t i = 0; i < n; ++i)
                dst[i] = (uint16_t)((lit[i] & 0x7Fu) | ((lit[i] >> 7) << 15) | (ex[i] << 7));
        }
    }
    free(active);
    free(lit);
    free(ex);
    return rc;
}

/* radix_pack.py:376-411 — per block, byte (k-1) of a uint16 is the word
 * length of nonterminal tier k's stream (k >= 1); a word past the payload
 * reads as zero (the device pad). Only meaningful for three or more tiers. */
int oracle_schedule(int64_t R, int64_t C, int64_t B, const int32_t *widths, int32_t nw,
                    const uint32_t *offsets, const uint32_t *data, int64_t nwords, uint16_t *out) {
    int64_t per_row = (C + B - 1) / B, nb = R * per_row;
    int32_t *rank = (int32_t *)malloc(sizeof(int32_t) * (size_t)B);
    for (int64_t blk = 0; blk < nb; ++blk) {
        int64_t n = C - (blk % per_row) * B;
        if (n > B) n = B;
        int64_t pos = (int64_t)offsets[blk] + ceil_words(n, MANT + 1);
        int64_t count = n;
        uint32_t header = 0;
        for (int64_t i = 0; i < n; ++i) rank[i] = (int32_t)i;
        for (int t = 0; t < nw - 1; ++t) {
            uint32_t w = (uint32_t)widths[t], esc = (1u << w) - 1;
            int64_t words = ceil_words(count, w);
            if (t > 0) header |= (uint32_t)words << ((t - 1) * 8);
            if (t < nw - 2) {
                int64_t kept = 0;
                for (int64_t i = 0; i < count; ++i) {
                    uint64_t bit = (uint64_t)i * w;
                    int64_t wi = pos + (int64_t)(bit >> 5);
                    uint32_t lo = (uint32_t)(bit & 31);
                    uint64_t a = wi < nwords ? data[wi] : 0, bb = wi + 1 < nwords ? data[wi + 1] : 0;
                    uint32_t code = (uint32_t)(((a >> lo) | (lo + w > 32 ? bb << (32 - lo) : 0)) & esc);
                    if (code == esc) ++kept;
                }
                count = kept;
            }
            pos += words;
        }
        out[blk] = (uint16_t)header;
    }
    free(rank);
    return 0;
}

static double bf16_to_double(uint16_t b) {
    uint32_t u = (uint32_t)b << 16;
    float f;
    memcpy(&f, &u, 4);
    return (double)f;
}

/* y[m, r] = sum_c x[m, c] * W[r, c] in float64, and the bound's
 * magnitude sum |x| @ |W|^T (bench/radix_gemv_bitpin.py:181-182). */
int oracle_linear_f64(int64_t M, int64_t R, int64_t C, const double *x, const uint16_t *w,
                      double *y, double *absy) {
    for (int64_t r = 0; r < R; ++r) {
        const uint16_t *row = w + r * C;
        for (int64_t m = 0; m < M; ++m) {
            const double *xm = x + m * C;
            double s = 0.0, a = 0.0;
            for (int64_t c = 0; c < C; ++c) {
                double wv = bf16_to_double(row[c]);
                s += xm[c] * wv;
                a += (xm[c] < 0 ? -xm[c] : xm[c]) * (wv < 0 ? -wv : wv);
            }
            y[m * R + r] = s;
            absy[m * R + r] = a;
        }
    }
    return 0;
}
