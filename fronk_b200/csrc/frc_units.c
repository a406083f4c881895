/* frc_units.c - unit files from disk, the way the reference node opens them
 * (src/units.c:25-75): a directory holds unit-BB.bin (one block's weights in
 * the reference byte layout) and unit-BB.sha256 (64 lowercase hex digits and
 * a newline).  The unit is mapped read-only (MAP_SHARED, as the reference
 * maps it), its SHA-256 checked against the recorded digest, and handed to
 * frc_load_unit, which copies it into HBM; the mapping is released after the
 * copy.  The reference's hash stamp cache (src/prep.c:37), paged blocks and
 * the unit transfer protocol belong to its storage layer and are not here.
 *
 * SHA-256 follows FIPS 180-4 (sections 4.1.2, 4.2.2, 5.1.1, 5.3.3, 6.2). */
#define _GNU_SOURCE
#include <errno.h>
#include <fcntl.h>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include "../../include/fronk_b200.h"
#include "frc_units.h"

/* ------------------------------------------------------------- SHA-256 */

/* FIPS 180-4 4.2.2: the first 32 bits of the fractional parts of the cube
 * roots of the first 64 primes. */
static const uint32_t kSha256K[64] = {
    0x428a2f98u, 0x71374491u, 0xb5c0fbcfu, 0xe9b5dba5u, 0x3956c25bu, 0x59f111f1u, 0x923f82a4u, 0xab1c5ed5u,
    0xd807aa98u, 0x12835b01u, 0x243185beu, 0x550c7dc3u, 0x72be5d74u, 0x80deb1feu, 0x9bdc06a7u, 0xc19bf174u,
    0xe49b69c1u, 0xefbe4786u, 0x0fc19dc6u, 0x240ca1ccu, 0x2de92c6fu, 0x4a7484aau, 0x5cb0a9dcu, 0x76f988dau,
    0x983e5152u, 0xa831c66du, 0xb00327c8u, 0xbf597fc7u, 0xc6e00bf3u, 0xd5a79147u, 0x06ca6351u, 0x14292967u,
    0x27b70a85u, 0x2e1b2138u, 0x4d2c6dfcu, 0x53380d13u, 0x650a7354u, 0x766a0abbu, 0x81c2c92eu, 0x92722c85u,
    0xa2bfe8a1u, 0xa81a664bu, 0xc24b8b70u, 0xc76c51a3u, 0xd192e819u, 0xd6990624u, 0xf40e3585u, 0x106aa070u,
    0x19a4c116u, 0x1e376c08u, 0x2748774cu, 0x34b0bcb5u, 0x391c0cb3u, 0x4ed8aa4au, 0x5b9cca4fu, 0x682e6ff3u,
    0x748f82eeu, 0x78a5636fu, 0x84c87814u, 0x8cc70208u, 0x90befffau, 0xa4506cebu, 0xbef9a3f7u, 0xc67178f2u};

/* FIPS 180-4 5.3.3: the first 32 bits of the fractional parts of the square
 * roots of the first 8 primes. */
static const uint32_t kSha256H0[8] = {0x6a09e667u, 0xbb67ae85u, 0x3c6ef372u, 0xa54ff53au,
                                      0x510e527fu, 0x9b05688cu, 0x1f83d9abu, 0x5be0cd19u};

static inline uint32_t rotr32(uint32_t x, unsigned n) { return (x >> n) | (x << (32 - n)); }

/* One 512-bit block (FIPS 180-4 6.2.2). */
static void sha256_block(uint32_t h[8], const uint8_t *p) {
    uint32_t w[64];
    for (unsigned t = 0; t < 16; ++t)
        w[t] = (uint32_t)p[4 * t] << 24 | (uint32_t)p[4 * t + 1] << 16 | (uint32_t)p[4 * t + 2] << 8 | p[4 * t + 3];
    for (unsigned t = 16; t < 64; ++t) {
        const uint32_t s0 = rotr32(w[t - 15], 7) ^ rotr32(w[t - 15], 18) ^ (w[t - 15] >> 3);
        const uint32_t s1 = rotr32(w[t - 2], 17) ^ rotr32(w[t - 2], 19) ^ (w[t - 2] >> 10);
        w[t] = w[t - 16] + s0 + w[t - 7] + s1;
    }
    uint32_t a = h[0], b = h[1], c = h[2], d = h[3], e = h[4], f = h[5], g = h[6], k = h[7];
    for (unsigned t = 0; t < 64; ++t) {
        const uint32_t S1 = rotr32(e, 6) ^ rotr32(e, 11) ^ rotr32(e, 25);
        const uint32_t ch = (e & f) ^ (~e & g);
        const uint32_t t1 = k + S1 + ch + kSha256K[t] + w[t];
        const uint32_t S0 = rotr32(a, 2) ^ rotr32(a, 13) ^ rotr32(a, 22);
        const uint32_t maj = (a & b) ^ (a & c) ^ (b & c);
        const uint32_t t2 = S0 + maj;
        k = g; g = f; f = e; e = d + t1; d = c; c = b; b = a; a = t1 + t2;
    }
    h[0] += a; h[1] += b; h[2] += c; h[3] += d; h[4] += e; h[5] += f; h[6] += g; h[7] += k;
}

int frc_sha256(const void *data, size_t len, uint8_t out[32]) {
    if ((!data && len) || !out) return FRC_INVALID;
    const uint8_t *p = (const uint8_t *)data;
    uint32_t h[8];
    memcpy(h, kSha256H0, sizeof h);
    size_t n = len;
    for (; n >= 64; n -= 64, p += 64) sha256_block(h, p);
    /* padding (5.1.1): 0x80, zeros, the message length in bits, big-endian */
    uint8_t tail[128] = {0};
    memcpy(tail, p, n);
    tail[n] = 0x80;
    const size_t tl = n + 9 <= 64 ? 64 : 128;
    const uint64_t bits = (uint64_t)len * 8;
    for (unsigned i = 0; i < 8; ++i) tail[tl - 1 - i] = (uint8_t)(bits >> (8 * i));
    sha256_block(h, tail);
    if (tl == 128) sha256_block(h, tail + 64);
    for (unsigned i = 0; i < 8; ++i) {
        out[4 * i] = (uint8_t)(h[i] >> 24);
        out[4 * i + 1] = (uint8_t)(h[i] >> 16);
        out[4 * i + 2] = (uint8_t)(h[i] >> 8);
        out[4 * i + 3] = (uint8_t)h[i];
    }
    return FRC_OK;
}

/* --------------------------------------------------------------- files */

static int say(char *why, size_t why_len, int rc, const char *fmt, ...) {
    if (why && why_len) {
        va_list ap;
        va_start(ap, fmt);
        vsnprintf(why, why_len, fmt, ap);
        va_end(ap);
    }
    return rc;
}

int frc_unit_map(const char *directory, unsigned block, uint64_t want_bytes, int verify, const void **data,
                 size_t *len, char *why, size_t why_len) {
    if (!directory || !data || !len || block >= FRC_MAX_BLOCKS)
        return say(why, why_len, FRC_INVALID, "bad unit arguments");
    *data = NULL;
    *len = 0;
    char path[1024], wanted[66];
    int n = snprintf(path, sizeof path, "%s/unit-%02u.sha256", directory, block);
    if (n < 0 || n >= (int)sizeof path) return say(why, why_len, FRC_INVALID, "unit directory path too long");
    FILE *f = fopen(path, "rb");
    if (!f) return say(why, why_len, FRC_IO, "%s: %s", path, strerror(errno));
    const size_t got = fread(wanted, 1, sizeof wanted, f);
    const int ferr = ferror(f);
    fclose(f);
    /* 64 lowercase hex digits and a newline, nothing else (src/units.c:38-40) */
    if (ferr) return say(why, why_len, FRC_IO, "%s: read error", path);
    if (got != 65 || wanted[64] != '\n') return say(why, why_len, FRC_INVALID, "%s: not 64 hex digits and a newline", path);
    for (unsigned i = 0; i < 64; ++i)
        if (!((wanted[i] >= '0' && wanted[i] <= '9') || (wanted[i] >= 'a' && wanted[i] <= 'f')))
            return say(why, why_len, FRC_INVALID, "%s: not 64 hex digits and a newline", path);
    snprintf(path, sizeof path, "%s/unit-%02u.bin", directory, block);
    const int fd = open(path, O_RDONLY);
    if (fd < 0) return say(why, why_len, FRC_IO, "%s: %s", path, strerror(errno));
    struct stat st;
    if (fstat(fd, &st) || !S_ISREG(st.st_mode)) {
        close(fd);
        return say(why, why_len, FRC_IO, "%s: not a regular file", path);
    }
    if ((want_bytes && (uint64_t)st.st_size != want_bytes) || st.st_size <= 0) {
        close(fd);
        return say(why, why_len, FRC_IO, "%s: %lld bytes, a unit has %llu", path, (long long)st.st_size,
                   (unsigned long long)want_bytes);
    }
    const size_t bytes = (size_t)st.st_size;
    void *m = mmap(NULL, bytes, PROT_READ, MAP_SHARED, fd, 0);
    close(fd);
    if (m == MAP_FAILED) return say(why, why_len, FRC_IO, "%s: mmap: %s", path, strerror(errno));
    madvise(m, bytes, MADV_SEQUENTIAL);
    if (verify) {
        uint8_t digest[32];
        char actual[65];
        frc_sha256(m, bytes, digest);
        for (unsigned i = 0; i < 32; ++i) snprintf(actual + 2 * i, 3, "%02x", digest[i]);
        if (memcmp(actual, wanted, 64)) {
            munmap(m, bytes);
            return say(why, why_len, FRC_MISMATCH, "%s: SHA-256 %.64s, recorded %.64s", path, actual, wanted);
        }
    }
    *data = m;
    *len = bytes;
    return FRC_OK;
}

void frc_unit_unmap(const void *data, size_t len) {
    if (data && len) munmap((void *)data, len);
}

int frc_unit_verify(const char *directory, unsigned block, uint64_t unit_bytes, int verify) {
    const void *data;
    size_t len;
    const int rc = frc_unit_map(directory, block, unit_bytes, verify, &data, &len, NULL, 0);
    if (rc == FRC_OK) frc_unit_unmap(data, len);
    return rc;
}
