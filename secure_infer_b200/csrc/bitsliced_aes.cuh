// bitsliced_aes.cuh -- AES-128 counter-mode blocks, 32 at a time, in bit-planes.
//
// A thread encrypts the 32 counter blocks IV || BE32(v), v = 32 g .. 32 g + 31,
// of one counter group g.  Its state is 128 32-bit words, one per bit of the
// 16-byte block: plane (byte b, bit k) holds, in bit j, bit k of byte b of
// block j (k = 0 is the most significant bit, as the S-box circuit numbers
// them).  Because the group is aligned to the counter value, the input needs
// no transposition: the five low counter bits are the fixed patterns
// 0xAAAAAAAA, 0xCCCCCCCC, 0xF0F0F0F0, 0xFF00FF00, 0xFFFF0000 and every other
// input plane is all zeros or all ones.
//
// Rounds (FIPS-197 5.1): SubBytes is bs_sbox on the eight planes of each byte;
// ShiftRows rotates the planes of rows 1-3 between columns (register moves);
// MixColumns works on the planes of a column, with xtime as a rewiring plus
// three XORs; AddRoundKey XORs each plane with a mask that is all ones where
// the round-key bit is set (rk_mask, 11 x 128 words, built once per CTA from
// the key schedule).  Rounds 1-9 run as a loop over one round body: unrolled,
// the ten rounds are about 25k instructions and the kernel stalls on
// instruction fetch.  A 32 x 32 bit transpose per output word brings each
// block back to byte order.  Byte b of the block is row b mod 4, column b / 4.
//
// Everything is __host__ __device__ so the CPU tests can run the same code.
#pragma once

#include <cstdint>

#include "bitsliced_sbox.cuh"

namespace sib {

// Round-key masks: rk_mask[(round * 16 + byte) * 8 + bit] for the 176 round-key
// bytes (byte order of FIPS-197, round keys one after the other).
SIB_HD void bs_round_key_masks(const uint8_t rk_bytes[176], uint32_t rk_mask[1408])
{
    for (int i = 0; i < 176; ++i)
        for (int k = 0; k < 8; ++k) rk_mask[i * 8 + k] = ((rk_bytes[i] >> (7 - k)) & 1u) ? 0xffffffffu : 0u;
}

// The 128 input planes of counter group g after AddRoundKey 0.  iv: the
// big-endian packs of the 12 fixed IV bytes (iv[0] holds bytes 0..3).
SIB_HD void bs_load_group(uint32_t st[16][8], const uint32_t iv[3], uint32_t g, const uint32_t* rk_mask)
{
    constexpr uint32_t kLow[5] = {0xAAAAAAAAu, 0xCCCCCCCCu, 0xF0F0F0F0u, 0xFF00FF00u, 0xFFFF0000u};
#pragma unroll
    for (int b = 0; b < 16; ++b) {
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            uint32_t plane;
            if (b < 12) {
                const uint32_t byte = (iv[b >> 2] >> (24 - 8 * (b & 3))) & 0xffu;
                plane = ((byte >> (7 - k)) & 1u) ? 0xffffffffu : 0u;
            } else {
                const int p = 8 * (15 - b) + (7 - k);   // bit of the counter value v
                plane = p < 5 ? kLow[p < 5 ? p : 0] : (((g >> (p - 5)) & 1u) ? 0xffffffffu : 0u);
            }
            st[b][k] = plane ^ rk_mask[b * 8 + k];
        }
    }
}

SIB_HD void bs_sub_bytes(uint32_t st[16][8])
{
#pragma unroll
    for (int b = 0; b < 16; ++b)
        bs_sbox(st[b][0], st[b][1], st[b][2], st[b][3], st[b][4], st[b][5], st[b][6], st[b][7], st[b][0], st[b][1],
                st[b][2], st[b][3], st[b][4], st[b][5], st[b][6], st[b][7]);
}

// ShiftRows: row r of the state moves r columns to the left.
SIB_HD void bs_shift_rows(uint32_t st[16][8])
{
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const uint32_t r1 = st[1][k];
        st[1][k] = st[5][k]; st[5][k] = st[9][k]; st[9][k] = st[13][k]; st[13][k] = r1;
        const uint32_t r2a = st[2][k], r2b = st[6][k];
        st[2][k] = st[10][k]; st[6][k] = st[14][k]; st[10][k] = r2a; st[14][k] = r2b;
        const uint32_t r3 = st[15][k];
        st[15][k] = st[11][k]; st[11][k] = st[7][k]; st[7][k] = st[3][k]; st[3][k] = r3;
    }
}

// MixColumns + AddRoundKey with the round key's 128 masks `key`:
// b_r = xtime(a_r ^ a_{r+1}) ^ a_r ^ (a_0 ^ a_1 ^ a_2 ^ a_3) ^ key.
SIB_HD void bs_mix_add(uint32_t st[16][8], const uint32_t* key)
{
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        uint32_t sum[8], a0[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            sum[k] = st[4 * c][k] ^ st[4 * c + 1][k] ^ st[4 * c + 2][k] ^ st[4 * c + 3][k];
            a0[k] = st[4 * c][k];
        }
        // Rows in order, each overwriting its own slot: row r still sees the
        // original row r + 1 (row 3 pairs with the saved row 0).
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            uint32_t t[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) t[k] = st[4 * c + r][k] ^ (r == 3 ? a0[k] : st[4 * c + r + 1][k]);
            // xtime on planes (k = 0 is bit 7): shift left, reduce by 0x1b.
            const uint32_t x[8] = {t[1], t[2], t[3], t[4] ^ t[0], t[5] ^ t[0], t[6], t[7] ^ t[0], t[0]};
#pragma unroll
            for (int k = 0; k < 8; ++k) st[4 * c + r][k] ^= x[k] ^ sum[k] ^ key[(4 * c + r) * 8 + k];
        }
    }
}

SIB_HD void bs_add_key(uint32_t st[16][8], const uint32_t* key)
{
#pragma unroll
    for (int b = 0; b < 16; ++b)
#pragma unroll
        for (int k = 0; k < 8; ++k) st[b][k] ^= key[b * 8 + k];
}

SIB_HD void bs_encrypt(uint32_t st[16][8], const uint32_t* rk_mask)
{
#pragma unroll 1
    for (int round = 1; round < 10; ++round) {
        bs_sub_bytes(st);
        bs_shift_rows(st);
        bs_mix_add(st, rk_mask + round * 128);
    }
    bs_sub_bytes(st);
    bs_shift_rows(st);
    bs_add_key(st, rk_mask + 1280);
}

// Transpose of a 32 x 32 bit matrix in place: afterwards bit m of a[j] is
// what bit j of a[m] was (recursive block swaps, 5 levels).
SIB_HD void bs_transpose32(uint32_t a[32])
{
    uint32_t m = 0x0000ffffu;
#pragma unroll
    for (int s = 16; s > 0; s >>= 1, m ^= m << s) {
#pragma unroll
        for (int k = 0; k < 32; k = (k + s + 1) & ~s) {
            const uint32_t t = ((a[k] >> s) ^ a[k + s]) & m;
            a[k] ^= t << s;
            a[k + s] ^= t;
        }
    }
}

// Little-endian output word w (bytes 4w .. 4w + 3) of the 32 blocks: out[j] is
// word w of block j.
template <int W>
SIB_HD void bs_store_word(const uint32_t st[16][8], uint32_t out[32])
{
#pragma unroll
    for (int t = 0; t < 4; ++t)
#pragma unroll
        for (int i = 0; i < 8; ++i) out[8 * t + i] = st[4 * W + t][7 - i];
    bs_transpose32(out);
}

}  // namespace sib
