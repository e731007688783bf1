// kx.cuh -- X25519 (RFC 7748) and BLAKE2b (RFC 7693) for the session key
// agreement (secure_infer.cpp:449-521, key_agreement.aicpu).  Shared by the
// device kernel and the host side of the handshake, so both ends run the same
// arithmetic.  Straight-line, single-thread code: a handshake runs once per
// session.  Field elements mod p = 2^255 - 19 use five 51-bit limbs.
#pragma once

#include <cstdint>

#ifdef __CUDACC__
#define KX_FN __host__ __device__ inline
#else
#define KX_FN inline
#endif

namespace kx {

// ---------------------------------------------------------------- BLAKE2b
struct Blake2b {
    uint64_t h[8];
    uint64_t t;           // bytes compressed so far
    uint8_t buf[128];
    uint32_t used;
    uint32_t outlen;
};

KX_FN uint64_t rotr64(uint64_t x, int n) { return (x >> n) | (x << (64 - n)); }

KX_FN uint64_t load64le(const uint8_t* p)
{
    uint64_t v = 0;
    for (int i = 7; i >= 0; --i) v = (v << 8) | p[i];
    return v;
}

KX_FN void blake2b_compress(Blake2b& s, const uint8_t block[128], bool last)
{
    // RFC 7693 section 2.6 / 3.2: IV (the SHA-512 initial values) and the
    // message schedule permutations.
    const uint64_t iv[8] = {0x6a09e667f3bcc908ull, 0xbb67ae8584caa73bull, 0x3c6ef372fe94f82bull,
                            0xa54ff53a5f1d36f1ull, 0x510e527fade682d1ull, 0x9b05688c2b3e6c1full,
                            0x1f83d9abfb41bd6bull, 0x5be0cd19137e2179ull};
    const uint8_t sigma[10][16] = {
        {0, 1, 2, 3, 4, 5, 6, 7, 8, 9, 10, 11, 12, 13, 14, 15}, {14, 10, 4, 8, 9, 15, 13, 6, 1, 12, 0, 2, 11, 7, 5, 3},
        {11, 8, 12, 0, 5, 2, 15, 13, 10, 14, 3, 6, 7, 1, 9, 4}, {7, 9, 3, 1, 13, 12, 11, 14, 2, 6, 5, 10, 4, 0, 15, 8},
        {9, 0, 5, 7, 2, 4, 10, 15, 14, 1, 11, 12, 6, 8, 3, 13}, {2, 12, 6, 10, 0, 11, 8, 3, 4, 13, 7, 5, 15, 14, 1, 9},
        {12, 5, 1, 15, 14, 13, 4, 10, 0, 7, 6, 3, 9, 2, 8, 11}, {13, 11, 7, 14, 12, 1, 3, 9, 5, 0, 15, 4, 8, 6, 2, 10},
        {6, 15, 14, 9, 11, 3, 0, 8, 12, 2, 13, 7, 1, 4, 10, 5}, {10, 2, 8, 4, 7, 6, 1, 5, 15, 11, 9, 14, 3, 12, 13, 0}};
    uint64_t m[16], v[16];
    for (int i = 0; i < 16; ++i) m[i] = load64le(block + 8 * i);
    for (int i = 0; i < 8; ++i) {
        v[i] = s.h[i];
        v[i + 8] = iv[i];
    }
    v[12] ^= s.t;            // 128-bit counter: messages here are far below 2^64 bytes
    if (last) v[14] = ~v[14];
    auto g = [&](int a, int b, int c, int d, uint64_t x, uint64_t y) {
        v[a] = v[a] + v[b] + x;
        v[d] = rotr64(v[d] ^ v[a], 32);
        v[c] = v[c] + v[d];
        v[b] = rotr64(v[b] ^ v[c], 24);
        v[a] = v[a] + v[b] + y;
        v[d] = rotr64(v[d] ^ v[a], 16);
        v[c] = v[c] + v[d];
        v[b] = rotr64(v[b] ^ v[c], 63);
    };
    for (int r = 0; r < 12; ++r) {
        const uint8_t* z = sigma[r % 10];
        g(0, 4, 8, 12, m[z[0]], m[z[1]]);
        g(1, 5, 9, 13, m[z[2]], m[z[3]]);
        g(2, 6, 10, 14, m[z[4]], m[z[5]]);
        g(3, 7, 11, 15, m[z[6]], m[z[7]]);
        g(0, 5, 10, 15, m[z[8]], m[z[9]]);
        g(1, 6, 11, 12, m[z[10]], m[z[11]]);
        g(2, 7, 8, 13, m[z[12]], m[z[13]]);
        g(3, 4, 9, 14, m[z[14]], m[z[15]]);
    }
    for (int i = 0; i < 8; ++i) s.h[i] ^= v[i] ^ v[i + 8];
}

KX_FN void blake2b_update(Blake2b& s, const uint8_t* in, uint64_t len)
{
    for (uint64_t i = 0; i < len; ++i) {
        if (s.used == 128) {       // a full buffer is compressed only once more input follows
            s.t += 128;
            blake2b_compress(s, s.buf, false);
            s.used = 0;
        }
        s.buf[s.used++] = in[i];
    }
}

// Keyed (key_len > 0) or plain BLAKE2b with an outlen-byte digest.
KX_FN void blake2b_init(Blake2b& s, uint32_t outlen, const uint8_t* key, uint32_t key_len)
{
    const uint64_t iv0 = 0x6a09e667f3bcc908ull;
    const uint64_t ivs[8] = {iv0, 0xbb67ae8584caa73bull, 0x3c6ef372fe94f82bull, 0xa54ff53a5f1d36f1ull,
                             0x510e527fade682d1ull, 0x9b05688c2b3e6c1full, 0x1f83d9abfb41bd6bull,
                             0x5be0cd19137e2179ull};
    for (int i = 0; i < 8; ++i) s.h[i] = ivs[i];
    s.h[0] ^= 0x01010000ull ^ (static_cast<uint64_t>(key_len) << 8) ^ outlen;
    s.t = 0;
    s.used = 0;
    s.outlen = outlen;
    if (key_len) {
        uint8_t block[128] = {};
        for (uint32_t i = 0; i < key_len; ++i) block[i] = key[i];
        blake2b_update(s, block, 128);
    }
}

KX_FN void blake2b_final(Blake2b& s, uint8_t* out)
{
    s.t += s.used;
    for (uint32_t i = s.used; i < 128; ++i) s.buf[i] = 0;
    blake2b_compress(s, s.buf, true);
    for (uint32_t i = 0; i < s.outlen; ++i) out[i] = static_cast<uint8_t>(s.h[i / 8] >> (8 * (i % 8)));
}

KX_FN void blake2b(uint8_t* out, uint32_t outlen, const uint8_t* key, uint32_t key_len, const uint8_t* in,
                   uint64_t len)
{
    Blake2b s;
    blake2b_init(s, outlen, key, key_len);
    blake2b_update(s, in, len);
    blake2b_final(s, out);
}

// ---------------------------------------------------------------- X25519
struct Fe {
    uint64_t v[5];
};

constexpr uint64_t kMask51 = (1ull << 51) - 1;

KX_FN void fe_carry(Fe& a)
{
    for (int r = 0; r < 2; ++r) {
        uint64_t c = 0;
        for (int i = 0; i < 5; ++i) {
            a.v[i] += c;
            c = a.v[i] >> 51;
            a.v[i] &= kMask51;
        }
        a.v[0] += 19 * c;
    }
}

KX_FN Fe fe_add(const Fe& a, const Fe& b)
{
    Fe r;
    for (int i = 0; i < 5; ++i) r.v[i] = a.v[i] + b.v[i];
    fe_carry(r);
    return r;
}

// a - b + 4p keeps every limb positive for reduced inputs.
KX_FN Fe fe_sub(const Fe& a, const Fe& b)
{
    Fe r;
    r.v[0] = a.v[0] + 0x1fffffffffffb4ull - b.v[0];
    for (int i = 1; i < 5; ++i) r.v[i] = a.v[i] + 0x1ffffffffffffcull - b.v[i];
    fe_carry(r);
    return r;
}

KX_FN Fe fe_mul(const Fe& a, const Fe& b)
{
    using u128 = unsigned __int128;
    const uint64_t b19[5] = {b.v[0] * 19, b.v[1] * 19, b.v[2] * 19, b.v[3] * 19, b.v[4] * 19};
    u128 t[5];
    t[0] = (u128)a.v[0] * b.v[0] + (u128)a.v[1] * b19[4] + (u128)a.v[2] * b19[3] + (u128)a.v[3] * b19[2] +
           (u128)a.v[4] * b19[1];
    t[1] = (u128)a.v[0] * b.v[1] + (u128)a.v[1] * b.v[0] + (u128)a.v[2] * b19[4] + (u128)a.v[3] * b19[3] +
           (u128)a.v[4] * b19[2];
    t[2] = (u128)a.v[0] * b.v[2] + (u128)a.v[1] * b.v[1] + (u128)a.v[2] * b.v[0] + (u128)a.v[3] * b19[4] +
           (u128)a.v[4] * b19[3];
    t[3] = (u128)a.v[0] * b.v[3] + (u128)a.v[1] * b.v[2] + (u128)a.v[2] * b.v[1] + (u128)a.v[3] * b.v[0] +
           (u128)a.v[4] * b19[4];
    t[4] = (u128)a.v[0] * b.v[4] + (u128)a.v[1] * b.v[3] + (u128)a.v[2] * b.v[2] + (u128)a.v[3] * b.v[1] +
           (u128)a.v[4] * b.v[0];
    Fe r;
    uint64_t c = 0;
    for (int i = 0; i < 5; ++i) {
        t[i] += c;
        r.v[i] = static_cast<uint64_t>(t[i]) & kMask51;
        c = static_cast<uint64_t>(t[i] >> 51);
    }
    r.v[0] += 19 * c;
    fe_carry(r);
    return r;
}

KX_FN Fe fe_mul_small(const Fe& a, uint64_t k)
{
    Fe r;
    uint64_t c = 0;
    for (int i = 0; i < 5; ++i) {
        const unsigned __int128 p = (unsigned __int128)a.v[i] * k + c;
        r.v[i] = static_cast<uint64_t>(p) & kMask51;
        c = static_cast<uint64_t>(p >> 51);
    }
    r.v[0] += 19 * c;
    fe_carry(r);
    return r;
}

// a^(p-2) = a^-1 (Fermat), p - 2 = 2^255 - 21: square-and-multiply over its bits.
KX_FN Fe fe_invert(const Fe& a)
{
    Fe r = a;   // bit 254 is set
    for (int i = 253; i >= 0; --i) {
        r = fe_mul(r, r);
        // 2^255 - 21 in binary: bits 254..5 set, bits 4..0 = 01011
        const bool bit = i >= 5 ? true : ((0x0bu >> i) & 1u) != 0;
        if (bit) r = fe_mul(r, a);
    }
    return r;
}

KX_FN Fe fe_frombytes(const uint8_t s[32])
{
    uint64_t w[4];
    for (int i = 0; i < 4; ++i) w[i] = load64le(s + 8 * i);
    w[3] &= 0x7fffffffffffffffull;   // the top bit is ignored (RFC 7748 section 5)
    Fe r;
    r.v[0] = w[0] & kMask51;
    r.v[1] = ((w[0] >> 51) | (w[1] << 13)) & kMask51;
    r.v[2] = ((w[1] >> 38) | (w[2] << 26)) & kMask51;
    r.v[3] = ((w[2] >> 25) | (w[3] << 39)) & kMask51;
    r.v[4] = (w[3] >> 12) & kMask51;
    return r;
}

KX_FN void fe_tobytes(uint8_t out[32], Fe a)
{
    fe_carry(a);
    // Full reduction: subtract p when a >= p.
    uint64_t q = (a.v[0] + 19) >> 51;
    for (int i = 1; i < 5; ++i) q = (a.v[i] + q) >> 51;
    a.v[0] += 19 * q;
    uint64_t c = 0;
    for (int i = 0; i < 5; ++i) {
        a.v[i] += c;
        c = a.v[i] >> 51;
        a.v[i] &= kMask51;
    }
    const uint64_t w[4] = {a.v[0] | (a.v[1] << 51), (a.v[1] >> 13) | (a.v[2] << 38), (a.v[2] >> 26) | (a.v[3] << 25),
                           (a.v[3] >> 39) | (a.v[4] << 12)};
    for (int i = 0; i < 32; ++i) out[i] = static_cast<uint8_t>(w[i / 8] >> (8 * (i % 8)));
}

KX_FN void fe_cswap(Fe& a, Fe& b, uint64_t swap)
{
    const uint64_t m = 0 - swap;
    for (int i = 0; i < 5; ++i) {
        const uint64_t x = m & (a.v[i] ^ b.v[i]);
        a.v[i] ^= x;
        b.v[i] ^= x;
    }
}

// RFC 7748 section 5: X25519(k, u) with the Montgomery ladder.
KX_FN void x25519(uint8_t out[32], const uint8_t scalar[32], const uint8_t point[32])
{
    uint8_t k[32];
    for (int i = 0; i < 32; ++i) k[i] = scalar[i];
    k[0] &= 248;
    k[31] &= 127;
    k[31] |= 64;
    const Fe x1 = fe_frombytes(point);
    Fe x2 = {{1, 0, 0, 0, 0}}, z2 = {{0, 0, 0, 0, 0}}, x3 = x1, z3 = {{1, 0, 0, 0, 0}};
    uint64_t swap = 0;
    for (int t = 254; t >= 0; --t) {
        const uint64_t kt = (k[t >> 3] >> (t & 7)) & 1u;
        swap ^= kt;
        fe_cswap(x2, x3, swap);
        fe_cswap(z2, z3, swap);
        swap = kt;
        const Fe a = fe_add(x2, z2), aa = fe_mul(a, a);
        const Fe b = fe_sub(x2, z2), bb = fe_mul(b, b);
        const Fe e = fe_sub(aa, bb);
        const Fe c = fe_add(x3, z3), d = fe_sub(x3, z3);
        const Fe da = fe_mul(d, a), cb = fe_mul(c, b);
        const Fe s1 = fe_add(da, cb), s2 = fe_sub(da, cb);
        x3 = fe_mul(s1, s1);
        z3 = fe_mul(x1, fe_mul(s2, s2));
        x2 = fe_mul(aa, bb);
        z2 = fe_mul(e, fe_add(aa, fe_mul_small(e, 121665)));
    }
    fe_cswap(x2, x3, swap);
    fe_cswap(z2, z3, swap);
    fe_tobytes(out, fe_mul(x2, fe_invert(z2)));
    for (int i = 0; i < 32; ++i) k[i] = 0;
}

KX_FN void x25519_public(uint8_t out[32], const uint8_t scalar[32])
{
    uint8_t base[32] = {9};
    x25519(out, scalar, base);
}

// The handshake's derivations (secure_infer.cpp:495-502, key_agreement.aicpu):
// key = BLAKE2b-128 keyed by the shared secret over info || host_public ||
// device_public || challenge; proof = BLAKE2b-256 keyed by the key over the
// challenge; IV salt = BLAKE2b-32 keyed by the shared secret over its label.
KX_FN void derive_key(uint8_t key[16], const uint8_t shared[32], const uint8_t host_public[32],
                      const uint8_t device_public[32], const uint8_t challenge[32])
{
    const char info[] = "SecureInfer X25519 BLAKE2b test v1";
    Blake2b s;
    blake2b_init(s, 16, shared, 32);
    blake2b_update(s, reinterpret_cast<const uint8_t*>(info), sizeof(info) - 1);
    blake2b_update(s, host_public, 32);
    blake2b_update(s, device_public, 32);
    blake2b_update(s, challenge, 32);
    blake2b_final(s, key);
}

KX_FN void derive_proof(uint8_t proof[32], const uint8_t key[16], const uint8_t challenge[32])
{
    blake2b(proof, 32, key, 16, challenge, 32);
}

KX_FN void derive_salt(uint8_t salt[4], const uint8_t shared[32])
{
    const char label[] = "SecureInfer IV salt v1";
    blake2b(salt, 4, shared, 32, reinterpret_cast<const uint8_t*>(label), sizeof(label) - 1);
}

}  // namespace kx
