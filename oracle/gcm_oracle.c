/*
 * gcm_oracle.c -- TEST INFRASTRUCTURE ONLY (the checker, never the product).
 *
 * CPU restatement of the reference secure_infer authenticated KV transfer
 * arithmetic.  Only tests/, __graft_entry__.smoke() and bench.py's CPU
 * baseline / reference arm load this library.  The shipped path is the CUDA
 * library under secure_infer_b200/ and never calls into this file.
 *
 * What is restated, and from where (paths relative to the reference project):
 *   - AES-128 key expansion + block encryption: FIPS-197 mathematics; the
 *     reference uses ARMv8 AESE/AESMC (secure_infer/native/kernels/aicpu/
 *     ghash.aicpu:60-221).  The S-box is derived here from its definition
 *     (GF(2^8) inverse + affine map), not typed in.
 *   - GF(2^128) multiply: NIST SP 800-38D Algorithm 1 (bit-serial), the
 *     field the reference evaluates with PMULL (ghash.aicpu:228-333).
 *   - CTR counter block: IV words 0..2 big-endian, word 3 = running counter
 *     incremented per 16-byte block (ghash.aicpu:133-147, :175-221).
 *   - GHASH over AAD || C || len, AAD first, zero-padded partial blocks,
 *     len = BE64(aad*8) || BE64(bytes*8) (ghash.aicpu:624-635).
 *   - Kernel semantics incl. fail-closed masking and status 1/0:
 *       aes_ctr :517-535, keystream :537-554, keystream_batch :559-582,
 *       gcm_decrypt_verify :594-651, gcm_encrypt_tag :656-699,
 *       gcm_verify_xor :705-773, gcm_verify_only :780-827,
 *       gcm_verify_xor_batch :834-940, gcm_xor_only :948-976,
 *       ghash (flags FINALIZE/VERIFY/XOR_ON_SUCCESS) :978-1046,
 *       auth_gate :1051-1068.
 *   - Host side: IV derivation secure_infer/native/secure_infer.cpp:274-300,
 *     64-byte AAD secure_infer.cpp:730-775, record layout + OpenSSL
 *     EVP_aes_128_gcm encrypt secure_infer.cpp:6379-6388 / :6508-6537,
 *     host decrypt+verify secure_infer.cpp:2479-2501.  OpenSSL libcrypto is the
 *     reference's own dependency for these host steps (Makefile:15-22).
 */
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <pthread.h>
#include <openssl/evp.h>

#define ORC_API __attribute__((visibility("default")))

/* ---------------------------------------------------------------- AES-128 */

static uint8_t g_sbox[256];
static pthread_once_t g_sbox_once = PTHREAD_ONCE_INIT;

static uint8_t gf8_mul(uint8_t a, uint8_t b)
{
    uint8_t p = 0;
    for (int i = 0; i < 8; ++i) {
        if (b & 1) p ^= a;
        uint8_t hi = a & 0x80;
        a = (uint8_t)(a << 1);
        if (hi) a ^= 0x1b;           /* x^8 = x^4 + x^3 + x + 1 */
        b >>= 1;
    }
    return p;
}

static void build_sbox(void)
{
    for (int x = 0; x < 256; ++x) {
        uint8_t inv = 0;
        if (x != 0) {
            for (int y = 1; y < 256; ++y) {
                if (gf8_mul((uint8_t)x, (uint8_t)y) == 1) { inv = (uint8_t)y; break; }
            }
        }
        /* affine map: b_i ^ b_{i+4} ^ b_{i+5} ^ b_{i+6} ^ b_{i+7} ^ c_i, c = 0x63 */
        uint8_t s = 0;
        for (int i = 0; i < 8; ++i) {
            int bit = ((inv >> i) & 1) ^ ((inv >> ((i + 4) & 7)) & 1) ^
                      ((inv >> ((i + 5) & 7)) & 1) ^ ((inv >> ((i + 6) & 7)) & 1) ^
                      ((inv >> ((i + 7) & 7)) & 1) ^ ((0x63 >> i) & 1);
            s |= (uint8_t)(bit << i);
        }
        g_sbox[x] = s;
    }
}

ORC_API const uint8_t* orc_aes_sbox(void)
{
    pthread_once(&g_sbox_once, build_sbox);
    return g_sbox;
}

ORC_API void orc_aes128_expand(const uint8_t key[16], uint8_t rk[176])
{
    const uint8_t* sbox = orc_aes_sbox();
    memcpy(rk, key, 16);
    uint8_t rcon = 1;
    for (int i = 4; i < 44; ++i) {
        uint8_t t[4];
        memcpy(t, rk + 4 * (i - 1), 4);
        if (i % 4 == 0) {
            uint8_t t0 = t[0];
            t[0] = (uint8_t)(sbox[t[1]] ^ rcon);
            t[1] = sbox[t[2]];
            t[2] = sbox[t[3]];
            t[3] = sbox[t0];
            rcon = gf8_mul(rcon, 2);
        }
        for (int j = 0; j < 4; ++j) rk[4 * i + j] = (uint8_t)(rk[4 * (i - 4) + j] ^ t[j]);
    }
}

ORC_API void orc_aes128_block(const uint8_t rk[176], const uint8_t in[16], uint8_t out[16])
{
    const uint8_t* sbox = orc_aes_sbox();
    uint8_t s[16];
    for (int i = 0; i < 16; ++i) s[i] = (uint8_t)(in[i] ^ rk[i]);
    for (int round = 1; round <= 10; ++round) {
        uint8_t t[16];
        /* SubBytes + ShiftRows: state is column-major, s[4c + r] */
        for (int c = 0; c < 4; ++c)
            for (int r = 0; r < 4; ++r)
                t[4 * c + r] = sbox[s[4 * ((c + r) & 3) + r]];
        if (round != 10) {
            for (int c = 0; c < 4; ++c) {
                uint8_t a0 = t[4 * c], a1 = t[4 * c + 1], a2 = t[4 * c + 2], a3 = t[4 * c + 3];
                s[4 * c + 0] = (uint8_t)(gf8_mul(a0, 2) ^ gf8_mul(a1, 3) ^ a2 ^ a3);
                s[4 * c + 1] = (uint8_t)(a0 ^ gf8_mul(a1, 2) ^ gf8_mul(a2, 3) ^ a3);
                s[4 * c + 2] = (uint8_t)(a0 ^ a1 ^ gf8_mul(a2, 2) ^ gf8_mul(a3, 3));
                s[4 * c + 3] = (uint8_t)(gf8_mul(a0, 3) ^ a1 ^ a2 ^ gf8_mul(a3, 2));
            }
        } else {
            memcpy(s, t, 16);
        }
        for (int i = 0; i < 16; ++i) s[i] ^= rk[16 * round + i];
    }
    memcpy(out, s, 16);
}

/* ------------------------------------------------------------ GF(2^128) */

/* SP 800-38D Algorithm 1.  Bit 0 of a block is the MSB of byte 0. */
ORC_API void orc_gf_mul(const uint8_t x[16], const uint8_t y[16], uint8_t out[16])
{
    uint8_t z[16] = {0}, v[16];
    memcpy(v, y, 16);
    for (int i = 0; i < 128; ++i) {
        if ((x[i >> 3] >> (7 - (i & 7))) & 1)
            for (int j = 0; j < 16; ++j) z[j] ^= v[j];
        int lsb = v[15] & 1;
        for (int j = 15; j > 0; --j) v[j] = (uint8_t)((v[j] >> 1) | (v[j - 1] << 7));
        v[0] >>= 1;
        if (lsb) v[0] ^= 0xe1;
    }
    memcpy(out, z, 16);
}

static void ghash_update(uint8_t state[16], const uint8_t h[16], const uint8_t* data, uint64_t bytes)
{
    for (uint64_t off = 0; off < bytes; off += 16) {
        uint64_t take = bytes - off < 16 ? bytes - off : 16;
        for (uint64_t i = 0; i < take; ++i) state[i] ^= data[off + i];
        orc_gf_mul(state, h, state);
    }
}

static void store_be64(uint8_t* out, uint64_t v)
{
    for (int i = 0; i < 8; ++i) out[i] = (uint8_t)(v >> (56 - 8 * i));
}

static void store_be32(uint8_t* out, uint32_t v)
{
    out[0] = (uint8_t)(v >> 24); out[1] = (uint8_t)(v >> 16);
    out[2] = (uint8_t)(v >> 8);  out[3] = (uint8_t)v;
}

/* S = GHASH_H(AAD || C || len) before the E_K(J0) mask. */
ORC_API void orc_ghash(const uint8_t h[16], const uint8_t* aad, uint64_t aad_bytes,
                       const uint8_t* c, uint64_t c_bytes, uint8_t out[16])
{
    uint8_t state[16] = {0}, len[16];
    if (aad_bytes) ghash_update(state, h, aad, aad_bytes);
    ghash_update(state, h, c, c_bytes);
    store_be64(len, aad_bytes * 8u);
    store_be64(len + 8, c_bytes * 8u);
    ghash_update(state, h, len, 16);
    memcpy(out, state, 16);
}

/* --------------------------------------------------- kernel semantics */

static void counter_block(uint8_t out[16], const uint32_t iv[4], uint32_t counter)
{
    for (int w = 0; w < 3; ++w) store_be32(out + 4 * w, iv[w]);
    store_be32(out + 12, counter);
}

static void ctr_process(const uint8_t* in, uint8_t* out, uint64_t bytes,
                        const uint8_t rk[176], const uint32_t iv[4])
{
    uint32_t counter = iv[3];
    for (uint64_t off = 0; off < bytes; off += 16, ++counter) {
        uint8_t cb[16], ks[16];
        counter_block(cb, iv, counter);
        orc_aes128_block(rk, cb, ks);
        uint64_t take = bytes - off < 16 ? bytes - off : 16;
        for (uint64_t i = 0; i < take; ++i) out[off + i] = in ? (uint8_t)(in[off + i] ^ ks[i]) : ks[i];
    }
}

static void tag_mask(const uint8_t rk[176], const uint32_t iv[4], uint8_t mask[16])
{
    uint8_t j0[16];
    counter_block(j0, iv, 1u);
    orc_aes128_block(rk, j0, mask);
}

static uint32_t tag_matches(const uint8_t s[16], const uint8_t mask[16], const uint8_t expected[16])
{
    uint8_t diff = 0;
    for (int i = 0; i < 16; ++i) diff |= (uint8_t)((s[i] ^ mask[i]) ^ expected[i]);
    return diff == 0 ? 1u : 0u;
}

ORC_API int orc_aes_ctr(const uint8_t* in, const uint8_t key[16], uint8_t* out,
                        uint64_t bytes, const uint32_t iv[4])
{
    if (!in || !key || !out || bytes == 0) return -1;
    uint8_t rk[176];
    orc_aes128_expand(key, rk);
    ctr_process(in, out, bytes, rk, iv);
    return 0;
}

ORC_API int orc_keystream(const uint8_t key[16], uint8_t* out, uint64_t bytes, const uint32_t iv[4])
{
    if (!key || !out || bytes == 0) return -1;
    uint8_t rk[176];
    orc_aes128_expand(key, rk);
    ctr_process(NULL, out, bytes, rk, iv);
    return 0;
}

ORC_API int orc_gcm_decrypt_verify(const uint8_t* c, const uint8_t key[16], const uint8_t h[16],
                                   const uint8_t tag[16], uint8_t* out, uint32_t* status,
                                   uint64_t bytes, const uint32_t iv[4],
                                   const uint8_t* aad, uint64_t aad_bytes)
{
    if (!c || !key || !h || !tag || !out || !status || bytes == 0 || (aad_bytes && !aad)) return -1;
    uint8_t rk[176], mask[16], s[16];
    orc_aes128_expand(key, rk);
    tag_mask(rk, iv, mask);
    orc_ghash(h, aad, aad_bytes, c, bytes, s);
    uint32_t ok = tag_matches(s, mask, tag);
    ctr_process(c, out, bytes, rk, iv);     /* always runs CTR: no timing oracle */
    uint8_t m = (uint8_t)(0u - ok);
    for (uint64_t i = 0; i < bytes; ++i) out[i] &= m;
    *status = ok;
    return 0;
}

ORC_API int orc_gcm_verify_xor(const uint8_t* c, const uint8_t key[16], const uint8_t h[16],
                               const uint8_t tag[16], const uint8_t* ks, uint8_t* out,
                               uint32_t* status, uint64_t bytes, const uint32_t iv[4],
                               const uint8_t* aad, uint64_t aad_bytes)
{
    if (!c || !key || !h || !tag || !ks || !out || !status || bytes == 0 || (aad_bytes && !aad)) return -1;
    uint8_t rk[176], mask[16], s[16];
    orc_aes128_expand(key, rk);
    tag_mask(rk, iv, mask);
    orc_ghash(h, aad, aad_bytes, c, bytes, s);
    uint32_t ok = tag_matches(s, mask, tag);
    uint8_t m = (uint8_t)(0u - ok);
    for (uint64_t i = 0; i < bytes; ++i) out[i] = (uint8_t)((c[i] ^ ks[i]) & m);
    *status = ok;
    return 0;
}

ORC_API int orc_gcm_verify_only(const uint8_t* c, const uint8_t key[16], const uint8_t h[16],
                                const uint8_t tag[16], uint32_t* status, uint64_t bytes,
                                const uint32_t iv[4], const uint8_t* aad, uint64_t aad_bytes)
{
    if (!c || !key || !h || !tag || !status || bytes == 0 || (aad_bytes && !aad)) return -1;
    uint8_t rk[176], mask[16], s[16];
    orc_aes128_expand(key, rk);
    tag_mask(rk, iv, mask);
    orc_ghash(h, aad, aad_bytes, c, bytes, s);
    *status = tag_matches(s, mask, tag);
    return 0;
}

ORC_API int orc_gcm_encrypt_tag(const uint8_t* p, const uint8_t key[16], const uint8_t h[16],
                                uint8_t* c_out, uint8_t tag_out[16], uint64_t bytes,
                                const uint32_t iv[4], const uint8_t* aad, uint64_t aad_bytes)
{
    if (!p || !key || !h || !c_out || !tag_out || bytes == 0 || (aad_bytes && !aad)) return -1;
    uint8_t rk[176], mask[16], s[16];
    orc_aes128_expand(key, rk);
    ctr_process(p, c_out, bytes, rk, iv);
    tag_mask(rk, iv, mask);
    orc_ghash(h, aad, aad_bytes, c_out, bytes, s);
    for (int i = 0; i < 16; ++i) tag_out[i] = (uint8_t)(s[i] ^ mask[i]);
    return 0;
}

enum { ORC_FINALIZE = 1, ORC_VERIFY = 2, ORC_XOR_ON_SUCCESS = 4 };

ORC_API int orc_ghash_flags(const uint8_t* in, const uint8_t h[16], uint8_t out[16],
                            const uint8_t* aad, const uint8_t* mask, const uint8_t* expected,
                            const uint8_t* ks, uint8_t* plain_out, uint32_t* status,
                            uint64_t in_bytes, uint64_t aad_bytes, uint32_t flags)
{
    if (!in || !h || !out || in_bytes == 0) return -1;
    if (aad_bytes && !aad) return -1;
    uint8_t s[16];
    orc_ghash(h, aad, aad_bytes, in, in_bytes, s);
    if (flags & ORC_FINALIZE) {
        if (!mask) return -1;
        for (int i = 0; i < 16; ++i) s[i] ^= mask[i];
    }
    memcpy(out, s, 16);
    uint32_t ok = 1;
    if (flags & ORC_VERIFY) {
        if (!expected) return -1;
        uint8_t diff = 0;
        for (int i = 0; i < 16; ++i) diff |= (uint8_t)(s[i] ^ expected[i]);
        ok = diff == 0;
    }
    if (flags & ORC_XOR_ON_SUCCESS) {
        if (!ks || !plain_out) return -1;
        uint8_t m = (uint8_t)(0u - ok);
        for (uint64_t i = 0; i < in_bytes; ++i) plain_out[i] = (uint8_t)((in[i] ^ ks[i]) & m);
    }
    if (status) *status = ok;
    return 0;
}

ORC_API int orc_auth_gate(uint8_t* data, const uint32_t* status, uint64_t bytes)
{
    if (!data || !status || bytes == 0) return -1;
    if (*status != 1u) memset(data, 0, bytes);
    return 0;
}

/* ------------------------------------------------------------ host side */

/* secure_infer.cpp:274-300.  In GCM mode the session nonce is 0
 * (secure_infer.cpp:242-245) and the counter base is 2. */
ORC_API void orc_derive_transfer_iv(const uint8_t base_iv[16], uint64_t session_nonce,
                                    uint64_t ticket, uint64_t block_offset, uint8_t out[16])
{
    memcpy(out, base_iv, 16);
    store_be64(out + 4, session_nonce + ticket);
    store_be32(out + 12, (uint32_t)(block_offset + 2u));
}

/* secure_infer.cpp:730-775 (after host-range lookup). */
ORC_API void orc_build_gcm_aad(uint8_t direction, uint32_t kind, uint32_t layer,
                               uint64_t block_id, uint64_t byte_offset, uint64_t bytes,
                               uint64_t ticket, uint64_t transfer_offset, uint64_t epoch,
                               uint8_t out[64])
{
    memset(out, 0, 64);
    out[0] = 'S'; out[1] = 'F'; out[2] = 'A'; out[3] = 'D';
    out[4] = 1;
    out[5] = direction;
    out[6] = (uint8_t)(kind & 0xffu);
    store_be32(out + 8, layer);
    store_be64(out + 12, block_id);
    store_be64(out + 20, byte_offset);
    store_be64(out + 28, bytes);
    store_be64(out + 36, ticket);
    store_be64(out + 44, transfer_offset);
    store_be64(out + 52, epoch);
}

ORC_API uint64_t orc_record_aligned_bytes(uint64_t count)
{
    uint64_t a = (count + 31u) & ~(uint64_t)31u;
    return a ? a : 32u;
}

ORC_API uint64_t orc_record_bytes(uint64_t count)
{
    return orc_record_aligned_bytes(count) + 32u + 64u;
}

/* Record = C (zero padded to 32) || tag16 || zero16 || AAD64
 * (secure_infer.cpp:6379-6388, :6508-6537).  OpenSSL EVP, IV length 12. */
ORC_API int orc_host_encrypt_record(const uint8_t key[16], const uint8_t iv[16],
                                    const uint8_t aad[64], const uint8_t* src,
                                    uint64_t count, uint8_t* record)
{
    const uint64_t aligned = orc_record_aligned_bytes(count);
    uint8_t aad_copy[64];
    if (aad) memcpy(aad_copy, aad, 64);   /* aad may live inside the record */
    memset(record, 0, aligned + 96u);
    EVP_CIPHER_CTX* ctx = EVP_CIPHER_CTX_new();
    if (!ctx) return -1;
    int n = 0, fin = 0, ok =
        EVP_EncryptInit_ex(ctx, EVP_aes_128_gcm(), NULL, NULL, NULL) == 1 &&
        EVP_CIPHER_CTX_ctrl(ctx, EVP_CTRL_GCM_SET_IVLEN, 12, NULL) == 1 &&
        EVP_EncryptInit_ex(ctx, NULL, NULL, key, iv) == 1;
    if (ok && aad) ok = EVP_EncryptUpdate(ctx, NULL, &n, aad_copy, 64) == 1;
    ok = ok && EVP_EncryptUpdate(ctx, record, &n, src, (int)count) == 1 &&
         EVP_EncryptFinal_ex(ctx, record + n, &fin) == 1 &&
         EVP_CIPHER_CTX_ctrl(ctx, EVP_CTRL_GCM_GET_TAG, 16, record + aligned) == 1;
    EVP_CIPHER_CTX_free(ctx);
    if (!ok) return -1;
    if (aad) memcpy(record + aligned + 32, aad_copy, 64);
    return 0;
}

/* secure_infer.cpp:2479-2501: DecryptInit -> AAD -> Update -> SET_TAG -> Final.
 * Returns 1 when authentic, 0 otherwise (output zeroed, as the reference's
 * failure path does), -1 on a setup error. */
ORC_API int orc_host_decrypt_verify(const uint8_t key[16], const uint8_t iv[16],
                                    const uint8_t* aad, const uint8_t* c, uint64_t count,
                                    const uint8_t tag[16], uint8_t* out)
{
    EVP_CIPHER_CTX* ctx = EVP_CIPHER_CTX_new();
    if (!ctx) return -1;
    int n = 0, fin = 0, ok =
        EVP_DecryptInit_ex(ctx, EVP_aes_128_gcm(), NULL, NULL, NULL) == 1 &&
        EVP_CIPHER_CTX_ctrl(ctx, EVP_CTRL_GCM_SET_IVLEN, 12, NULL) == 1 &&
        EVP_DecryptInit_ex(ctx, NULL, NULL, key, iv) == 1;
    if (ok && aad) ok = EVP_DecryptUpdate(ctx, NULL, &n, aad, 64) == 1;
    ok = ok && EVP_DecryptUpdate(ctx, out, &n, c, (int)count) == 1 &&
         EVP_CIPHER_CTX_ctrl(ctx, EVP_CTRL_GCM_SET_TAG, 16, (void*)tag) == 1 &&
         EVP_DecryptFinal_ex(ctx, out + n, &fin) == 1;
    EVP_CIPHER_CTX_free(ctx);
    if (!ok) memset(out, 0, count);
    return ok ? 1 : 0;
}

/* ---------------------------------------- multi-threaded CPU baseline */

typedef struct {
    const uint8_t* key;
    const uint8_t* ivs;        /* [n][16] */
    const uint8_t* records;    /* [n][stride] */
    uint64_t stride, count;
    uint8_t* const* outs;      /* [n] destinations */
    uint32_t* status;          /* [n] */
    uint64_t n;
    int encrypt;               /* 1: encrypt plaintext outs[i] into records[i] */
    int tid, nthreads;
} batch_job;

static void* batch_worker(void* arg)
{
    batch_job* job = (batch_job*)arg;
    const uint64_t aligned = orc_record_aligned_bytes(job->count);
    for (uint64_t i = (uint64_t)job->tid; i < job->n; i += (uint64_t)job->nthreads) {
        const uint8_t* rec = job->records + i * job->stride;
        if (job->encrypt) {
            job->status[i] = orc_host_encrypt_record(job->key, job->ivs + 16 * i,
                rec + aligned + 32, job->outs[i], job->count, (uint8_t*)rec) == 0;
        } else {
            job->status[i] = (uint32_t)orc_host_decrypt_verify(job->key, job->ivs + 16 * i,
                rec + aligned + 32, rec, job->count, rec + aligned, job->outs[i]);
        }
    }
    return NULL;
}

/* Decrypt+verify (encrypt=0) or encrypt (encrypt=1, AAD read from the record
 * slot, which the caller pre-fills) n records over nthreads POSIX threads. */
ORC_API int orc_host_batch(const uint8_t key[16], const uint8_t* ivs, const uint8_t* records,
                           uint64_t stride, uint64_t count, uint8_t* const* outs,
                           uint32_t* status, uint64_t n, int nthreads, int encrypt)
{
    if (nthreads < 1) nthreads = 1;
    if (nthreads > 256) nthreads = 256;
    pthread_t th[256];
    batch_job jobs[256];
    for (int t = 0; t < nthreads; ++t) {
        jobs[t] = (batch_job){key, ivs, records, stride, count, outs, status, n, encrypt, t, nthreads};
        if (t > 0 && pthread_create(&th[t], NULL, batch_worker, &jobs[t]) != 0) return -1;
    }
    batch_worker(&jobs[0]);
    for (int t = 1; t < nthreads; ++t) pthread_join(th[t], NULL);
    return 0;
}
