// gcm_device.cuh -- device primitives for the authenticated KV transfer path.
//
// AES-128 (FIPS-197) and GHASH (NIST SP 800-38D) for sm_100a.  Nothing here is
// a dense contraction: AES runs as shared-memory T-table lookups replicated
// per bank (lane l always reads bank l, so a warp never conflicts), and GHASH
// multiplies by a fixed power of H with 4-bit "nibble position" tables
// (32 positions x 16 values x 16 bytes = 8 KiB per power, reduction folded
// into the entries), replicated 8x so each quarter-warp of a 128-bit load is
// conflict-free.
//
// Word conventions.  Payload, keystream, AAD and tags are moved with 128-bit
// loads, so every 16-byte block lives in registers as four little-endian
// 32-bit words of its memory bytes ("LE layout").  AES round keys and T-tables
// use the same LE layout, so no byte swaps are needed on the hot path.  Table
// construction does its GF(2^128) shifts on big-endian words ("BE layout":
// word 0 = bytes 0..3, bit 31 of word 0 = coefficient of x^0) and swaps once
// when it stores an entry.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace sib {

// ----------------------------------------------------------------------------
// Compile-time AES tables, derived from the FIPS-197 definitions (GF(2^8)
// inverse modulo x^8+x^4+x^3+x+1 followed by the affine map with 0x63).
// ----------------------------------------------------------------------------
constexpr uint8_t gf8_mul_c(uint8_t a, uint8_t b)
{
    uint8_t p = 0;
    for (int i = 0; i < 8; ++i) {
        if (b & 1) p = static_cast<uint8_t>(p ^ a);
        const bool hi = (a & 0x80) != 0;
        a = static_cast<uint8_t>(a << 1);
        if (hi) a = static_cast<uint8_t>(a ^ 0x1b);
        b = static_cast<uint8_t>(b >> 1);
    }
    return p;
}

constexpr uint8_t gf8_inv_c(uint8_t x)
{
    // x^254 = x^-1 in GF(2^8) (and 0 -> 0).
    uint8_t result = 1, base = x;
    for (int e = 254; e; e >>= 1) {
        if (e & 1) result = gf8_mul_c(result, base);
        base = gf8_mul_c(base, base);
    }
    return x ? result : 0;
}

constexpr uint8_t sbox_c(uint8_t x)
{
    const uint8_t b = gf8_inv_c(x);
    uint8_t s = 0;
    for (int i = 0; i < 8; ++i) {
        const int bit = ((b >> i) ^ (b >> ((i + 4) & 7)) ^ (b >> ((i + 5) & 7)) ^
                         (b >> ((i + 6) & 7)) ^ (b >> ((i + 7) & 7)) ^ (0x63 >> i)) & 1;
        s = static_cast<uint8_t>(s | (bit << i));
    }
    return s;
}

struct AesTables {
    // te0[x] = MixColumns column of S(x) placed in row 0, LE word:
    // bytes (2*S, S, S, 3*S).  Rows 1..3 are rotations by 8/16/24.
    uint32_t te0[256];
};

constexpr AesTables make_aes_tables()
{
    AesTables t{};
    for (int x = 0; x < 256; ++x) {
        const uint8_t s = sbox_c(static_cast<uint8_t>(x));
        const uint32_t s1 = s, s2 = gf8_mul_c(s, 2), s3 = gf8_mul_c(s, 3);
        t.te0[x] = s2 | (s1 << 8) | (s1 << 16) | (s3 << 24);
    }
    return t;
}

constexpr AesTables kAesHost = make_aes_tables();
__device__ const AesTables kAesDev = kAesHost;

// ----------------------------------------------------------------------------
// Small helpers
// ----------------------------------------------------------------------------
__device__ __forceinline__ uint32_t bswap32(uint32_t x) { return __byte_perm(x, 0, 0x0123); }

__device__ __forceinline__ uint4 bswap4(uint4 v)
{
    return make_uint4(bswap32(v.x), bswap32(v.y), bswap32(v.z), bswap32(v.w));
}

__device__ __forceinline__ uint4 xor4(uint4 a, uint4 b)
{
    return make_uint4(a.x ^ b.x, a.y ^ b.y, a.z ^ b.z, a.w ^ b.w);
}

__device__ __forceinline__ uint4 zero4() { return make_uint4(0u, 0u, 0u, 0u); }

__device__ __forceinline__ bool is_zero4(uint4 v) { return (v.x | v.y | v.z | v.w) == 0u; }

__device__ __forceinline__ uint32_t rotl32(uint32_t x, int r) { return __funnelshift_l(x, x, r); }

// Read-only 16-byte load through the non-coherent path (inputs are never
// written by the kernel that reads them).
__device__ __forceinline__ uint4 ldg16(const uint8_t* p)
{
    return __ldg(reinterpret_cast<const uint4*>(p));
}

// Load up to 16 bytes (zero padded) from any alignment.
__device__ __forceinline__ uint4 load_partial16(const uint8_t* p, uint64_t avail)
{
    uint32_t w[4] = {0u, 0u, 0u, 0u};
    const int n = avail >= 16 ? 16 : static_cast<int>(avail);
    for (int i = 0; i < n; ++i) w[i >> 2] |= static_cast<uint32_t>(__ldg(p + i)) << (8 * (i & 3));
    return make_uint4(w[0], w[1], w[2], w[3]);
}

__device__ __forceinline__ void store_partial16(uint8_t* p, uint4 v, uint64_t avail)
{
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
    const int n = avail >= 16 ? 16 : static_cast<int>(avail);
    for (int i = 0; i < n; ++i) p[i] = static_cast<uint8_t>(w[i >> 2] >> (8 * (i & 3)));
}

// ----------------------------------------------------------------------------
// AES-128 in LE layout
// ----------------------------------------------------------------------------
__device__ __forceinline__ uint32_t aes_sbox_global(uint32_t x) { return (kAesDev.te0[x & 0xff] >> 8) & 0xffu; }

// Key expansion (FIPS-197 sec. 5.2) into 44 LE round-key words.  One thread.
__device__ inline void aes128_expand_le(const uint8_t* key, uint32_t rk[44])
{
    for (int i = 0; i < 4; ++i) {
        rk[i] = static_cast<uint32_t>(key[4 * i]) | (static_cast<uint32_t>(key[4 * i + 1]) << 8) |
                (static_cast<uint32_t>(key[4 * i + 2]) << 16) | (static_cast<uint32_t>(key[4 * i + 3]) << 24);
    }
    uint32_t rcon = 1;
    for (int i = 4; i < 44; ++i) {
        uint32_t t = rk[i - 1];
        if ((i & 3) == 0) {
            // RotWord is a right rotation by one byte in LE layout.
            t = (t >> 8) | (t << 24);
            t = aes_sbox_global(t) | (aes_sbox_global(t >> 8) << 8) |
                (aes_sbox_global(t >> 16) << 16) | (aes_sbox_global(t >> 24) << 24);
            t ^= rcon;
            rcon = (rcon << 1) ^ ((rcon & 0x80u) ? 0x11bu : 0u);
        }
        rk[i] = rk[i - 4] ^ t;
    }
}

// One AES-128 block.  `T(v)` returns te0[v] for a byte value v; the caller
// decides where the table lives (replicated shared memory on the hot path,
// global memory for one-off blocks).
template <class TableLookup, class RoundKey>
__device__ __forceinline__ uint4 aes128_encrypt_le(uint4 in, TableLookup T, RoundKey rk)
{
    uint32_t s0 = in.x ^ rk(0), s1 = in.y ^ rk(1), s2 = in.z ^ rk(2), s3 = in.w ^ rk(3);
#pragma unroll
    for (int r = 1; r < 10; ++r) {
        const uint32_t t0 = T(s0 & 0xff) ^ rotl32(T((s1 >> 8) & 0xff), 8) ^
                            rotl32(T((s2 >> 16) & 0xff), 16) ^ rotl32(T(s3 >> 24), 24) ^ rk(4 * r);
        const uint32_t t1 = T(s1 & 0xff) ^ rotl32(T((s2 >> 8) & 0xff), 8) ^
                            rotl32(T((s3 >> 16) & 0xff), 16) ^ rotl32(T(s0 >> 24), 24) ^ rk(4 * r + 1);
        const uint32_t t2 = T(s2 & 0xff) ^ rotl32(T((s3 >> 8) & 0xff), 8) ^
                            rotl32(T((s0 >> 16) & 0xff), 16) ^ rotl32(T(s1 >> 24), 24) ^ rk(4 * r + 2);
        const uint32_t t3 = T(s3 & 0xff) ^ rotl32(T((s0 >> 8) & 0xff), 8) ^
                            rotl32(T((s1 >> 16) & 0xff), 16) ^ rotl32(T(s2 >> 24), 24) ^ rk(4 * r + 3);
        s0 = t0; s1 = t1; s2 = t2; s3 = t3;
    }
    // Final round: SubBytes + ShiftRows only.  S(x) is byte 1 of te0[x].
    auto b0 = [&](uint32_t x) { return (T(x) >> 8) & 0x000000ffu; };
    auto b1 = [&](uint32_t x) { return T(x) & 0x0000ff00u; };
    auto b2 = [&](uint32_t x) { return (T(x) << 8) & 0x00ff0000u; };
    auto b3 = [&](uint32_t x) { return (T(x) << 16) & 0xff000000u; };
    uint4 out;
    out.x = (b0(s0 & 0xff) | b1((s1 >> 8) & 0xff) | b2((s2 >> 16) & 0xff) | b3(s3 >> 24)) ^ rk(40);
    out.y = (b0(s1 & 0xff) | b1((s2 >> 8) & 0xff) | b2((s3 >> 16) & 0xff) | b3(s0 >> 24)) ^ rk(41);
    out.z = (b0(s2 & 0xff) | b1((s3 >> 8) & 0xff) | b2((s0 >> 16) & 0xff) | b3(s1 >> 24)) ^ rk(42);
    out.w = (b0(s3 & 0xff) | b1((s0 >> 8) & 0xff) | b2((s1 >> 16) & 0xff) | b3(s2 >> 24)) ^ rk(43);
    return out;
}

// Counter block for 16-byte block index `c` of a payload whose IV words are
// big-endian packs of the IV bytes (word 3 = first counter, 2 for a GCM
// payload, 1 for J0).  The counter wraps modulo 2^32 like the reference's
// uint32 counter.
__device__ __forceinline__ uint4 ctr_block_le(const uint32_t iv[4], uint64_t c)
{
    return make_uint4(bswap32(iv[0]), bswap32(iv[1]), bswap32(iv[2]),
                      bswap32(iv[3] + static_cast<uint32_t>(c)));
}

// Shared-memory AES table replicated per bank: word (v * 32 + lane).
struct SmemAes {
    const uint32_t* te;   // [256][32]
    const uint32_t* rk;   // [44]
    uint32_t lane;
    __device__ __forceinline__ uint4 encrypt(uint4 in) const
    {
        const uint32_t* base = te + lane;
        return aes128_encrypt_le(
            in, [base](uint32_t v) { return base[v * 32u]; }, [this](int i) { return rk[i]; });
    }
};

// One-off AES block from global tables (finalisers, schedule build).
__device__ __forceinline__ uint4 aes128_encrypt_global(uint4 in, const uint32_t* rk)
{
    return aes128_encrypt_le(
        in, [](uint32_t v) { return kAesDev.te0[v]; }, [rk](int i) { return rk[i]; });
}

// ----------------------------------------------------------------------------
// GF(2^128)
// ----------------------------------------------------------------------------
// V * x^n for 1 <= n <= 32 in BE layout: shift right by n, then fold the n
// coefficients pushed past x^127 back with x^128 = 1 + x + x^2 + x^7.
__device__ __forceinline__ uint4 gf_mulx_n_be(uint4 v, int n)
{
    const uint32_t spill = v.w << (32 - n);
    uint4 r;
    r.w = __funnelshift_rc(v.w, v.z, n);
    r.z = __funnelshift_rc(v.z, v.y, n);
    r.y = __funnelshift_rc(v.y, v.x, n);
    r.x = n >= 32 ? 0u : (v.x >> n);
    r.x ^= spill ^ (spill >> 1) ^ (spill >> 2) ^ (spill >> 7);
    r.y ^= (spill << 31) ^ (spill << 30) ^ (spill << 25);
    return r;
}

// Nibble p (0..31, GCM bit order) of a block held in LE layout.
__device__ __forceinline__ uint32_t nibble_le(uint4 z, int p)
{
    const int byte = p >> 1;
    const int word = byte >> 2;
    const uint32_t w = word == 0 ? z.x : word == 1 ? z.y : word == 2 ? z.z : z.w;
    const int shift = (byte & 3) * 8 + ((p & 1) ? 0 : 4);
    return (w >> shift) & 0xfu;
}

// Z * M using M's nibble tables.  tab entry (p, v) lives at
// tab[(p * 16 + v) * kRep + rep]; kRep = 8 for the replicated shared-memory
// copy (rep = lane & 7), 1 for a global copy (rep = 0).
template <int kRep, bool kGlobal>
__device__ __forceinline__ uint4 gf_mul_table(uint4 z, const uint4* __restrict__ tab, uint32_t rep)
{
    uint4 acc0 = zero4(), acc1 = zero4();
#pragma unroll
    for (int p = 0; p < 32; p += 2) {
        const uint4* e0p = tab + (p * 16 + nibble_le(z, p)) * kRep + rep;
        const uint4* e1p = tab + ((p + 1) * 16 + nibble_le(z, p + 1)) * kRep + rep;
        const uint4 e0 = kGlobal ? __ldg(e0p) : *e0p;
        const uint4 e1 = kGlobal ? __ldg(e1p) : *e1p;
        acc0 = xor4(acc0, e0);
        acc1 = xor4(acc1, e1);
    }
    return xor4(acc0, acc1);
}

// Z * M using M's byte tables: entry (b, v) = v placed at byte b of a block,
// times M, stored at tab[((b >> 3) * 256 + v) * 8 + (b & 7)] (64 KiB, one
// copy).  At step s lane rep (= lane & 7) reads byte position s ^ rep, so the
// eight lanes of a shared-memory phase read eight distinct 16-byte bank groups:
// 16 conflict-free LDS.128 per product, half the shared-memory traffic of the
// nibble tables and no replication.
__device__ __forceinline__ uint4 gf_mul_byte8(uint4 z, const uint4* __restrict__ tab, uint32_t rep)
{
    // zp byte s = z byte (s ^ rep): swap word pairs for rep bit 2, then permute
    // bytes within each word for rep bits 0-1.
    const bool sw = (rep & 4u) != 0;
    const uint32_t sel = 0x3210u ^ (0x1111u * (rep & 3u));
    const uint32_t w[4] = {__byte_perm(sw ? z.y : z.x, 0u, sel), __byte_perm(sw ? z.x : z.y, 0u, sel),
                           __byte_perm(sw ? z.w : z.z, 0u, sel), __byte_perm(sw ? z.z : z.w, 0u, sel)};
    const char* base = reinterpret_cast<const char*>(tab);
    uint4 acc0 = zero4(), acc1 = zero4();
#pragma unroll
    for (int s = 0; s < 16; s += 2) {
        const uint32_t k0 = s & 3, k1 = (s + 1) & 3;
        const uint32_t v0 = k0 == 0 ? (w[s >> 2] << 7) : (w[s >> 2] >> (8 * k0 - 7));
        const uint32_t v1 = w[(s + 1) >> 2] >> (8 * k1 - 7);
        const uint32_t o0 = (v0 & 0x7f80u) | ((((s & 7) ^ rep)) << 4);
        const uint32_t o1 = (v1 & 0x7f80u) | (((((s + 1) & 7) ^ rep)) << 4);
        const uint4 e0 = *reinterpret_cast<const uint4*>(base + (s >> 3) * 32768 + o0);
        const uint4 e1 = *reinterpret_cast<const uint4*>(base + ((s + 1) >> 3) * 32768 + o1);
        acc0 = xor4(acc0, e0);
        acc1 = xor4(acc1, e1);
    }
    return xor4(acc0, acc1);
}

// Build the 32x16 nibble table of M (given in BE layout) cooperatively in one
// warp: lane p produces the 16 entries of nibble position p,
// T_p[v] = sum over bits of v of M * x^(4p + j) (bit 3 of v <-> j = 0).
// Entries are written in LE layout to dst[p * 16 + v].
__device__ inline void build_nibble_table_warp(uint4 m_be, uint4* dst, int lane)
{
    uint4 p0 = m_be;
    int k = 4 * lane;
    while (k >= 32) { p0 = gf_mulx_n_be(p0, 32); k -= 32; }
    if (k) p0 = gf_mulx_n_be(p0, k);
    const uint4 p1 = gf_mulx_n_be(p0, 1);
    const uint4 p2 = gf_mulx_n_be(p1, 1);
    const uint4 p3 = gf_mulx_n_be(p2, 1);
#pragma unroll
    for (int v = 0; v < 16; ++v) {
        uint4 e = zero4();
        if (v & 8) e = xor4(e, p0);
        if (v & 4) e = xor4(e, p1);
        if (v & 2) e = xor4(e, p2);
        if (v & 1) e = xor4(e, p3);
        dst[lane * 16 + v] = bswap4(e);
    }
}

// ----------------------------------------------------------------------------
// Per-session key schedule (device resident).
// ----------------------------------------------------------------------------
// A segment CTA of 256 threads hashes up to 16 blocks per thread with a
// Horner stride of H^256, giving 256 partials Y_t with
//   S_seg = sum_t Y_t * H^(256 - t),  t = 32 w + l,  256 - t = 32 (7 - w) + (32 - l).
// Each warp first scales its lanes by H^(32 (7 - w)), warps are XOR-combined,
// then lane l scales by H^(32 - l): every lane multiplies once, no idle lanes.
// CTA segments of one record are joined by Horner with H^kSegBlocks.
// The layer kernel gives each warp a segment of 32 k blocks (k = 1..64,
// chosen per launch so the segments fill the GPU's warps once), Horner stride
// H^32, a two-stage lane combine (lane 8q + r: H^(8 - r) then H^(24 - 8q)),
// and joins the segments with H^(32 k).
//   tab[e - 1]         H^e,      e = 1..32
//   tab[30 + k]        H^(32 k), k = 2..64  (tab[38] = H^256, the CTA stride)
//   tab[95]            H^4096 (CTA segment join)
// byte32 / lane8 hold shared-memory-ready copies: H^32 as byte tables (see
// gf_mul_byte8), and the eight nibble tables H^(8 - r) interleaved by r in
// the (p, v, r) layout.
constexpr int kGhashTables = 96;
constexpr int kThreads = 256;                       // threads per segment CTA
constexpr int kSegBlocks = 4096;                    // 16-byte blocks per segment
constexpr int kTabStride = 38;                      // H^256
constexpr int kTabSeg = 95;                         // H^4096
constexpr int kMaxWarpSegSteps = 64;                // layer kernel: segment <= 64 x 32 blocks

__host__ __device__ constexpr int tab_pow_small(int e) { return e - 1; }             // H^e, 1 <= e <= 32
__host__ __device__ constexpr int tab_pow_32k(int k) { return k == 1 ? 31 : 30 + k; }  // H^(32k), 1 <= k <= 64

struct __align__(16) GcmSchedule {
    uint32_t rk[44];          // AES-128 round keys, LE layout
    uint8_t key_copy[16];     // inputs the schedule was built from
    uint8_t h_copy[16];
    uint32_t valid;           // 1 once built
    uint32_t h_from_key;      // 1: H = E_K(0^128) derived on device
    uint32_t reserved[2];
    uint4 h_le;               // hash subkey H (memory bytes, LE words)
    uint4 tab[kGhashTables][32 * 16];
    uint4 byte32[2 * 256 * 8]; // H^32, byte position b, value v at [((b >> 3) * 256 + v) * 8 + (b & 7)]
    uint4 lane8[32 * 16 * 8]; // H^(8 - r) at [(p * 16 + v) * 8 + r], r = 0..7
    uint4 pow2hi[5][32 * 16]; // H^(2^e), e = 13..17 (segment joins of the plugin kernel)
    uint4 byte256[2 * 256 * 8]; // H^256 byte tables, layout of byte32 (Horner table of the plugin kernel)
};

// Nibble table of H^(2^e), 8 <= e <= 17.
__device__ __forceinline__ const uint4* tab_pow2(const GcmSchedule* S, int e)
{
    return e <= 11 ? S->tab[tab_pow_32k(1 << (e - 5))] : e == 12 ? S->tab[kTabSeg] : S->pow2hi[e - 13];
}

}  // namespace sib
