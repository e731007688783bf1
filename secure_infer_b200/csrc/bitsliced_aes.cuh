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
// ShiftRows moves no data -- after k rounds, logical byte (row r, column c) is
// kept in slot 4 ((c + k r) mod 4) + r, a compile-time index; MixColumns works
// on the planes of a column, with xtime as a rewiring plus three XORs, in place
// over the slots it reads; AddRoundKey XORs each plane with a mask that is all
// ones where the round-key bit is set (rk_mask, 11 x 128 words, built once per
// CTA from the key schedule).  A 32 x 32 bit transpose per output word brings
// each block back to byte order.
//
// Everything is __host__ __device__ so the CPU tests can run the same code.
#pragma once

#include <cstdint>

#include "bitsliced_sbox.cuh"

namespace sib {

// Slot of logical byte (row r, column c) after k ShiftRows.
SIB_HD constexpr int bs_slot(int r, int c, int k) { return 4 * ((c + k * r) & 3) + r; }

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

// MixColumns + AddRoundKey of round K (1..9), after that round's ShiftRows:
// column c holds logical rows r in slots bs_slot(r, c, K).
// b_r = xtime(a_r ^ a_{r+1}) ^ a_r ^ (a_0 ^ a_1 ^ a_2 ^ a_3) ^ key.
template <int K>
SIB_HD void bs_mix_add(uint32_t st[16][8], const uint32_t* rk_mask)
{
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        const int slot[4] = {bs_slot(0, c, K), bs_slot(1, c, K), bs_slot(2, c, K), bs_slot(3, c, K)};
        uint32_t sum[8], a0[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            sum[k] = st[slot[0]][k] ^ st[slot[1]][k] ^ st[slot[2]][k] ^ st[slot[3]][k];
            a0[k] = st[slot[0]][k];
        }
        // Rows in order, each overwriting its own slot: row r still sees the
        // original row r + 1 (row 3 pairs with the saved row 0).
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            uint32_t t[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) t[k] = st[slot[r]][k] ^ (r == 3 ? a0[k] : st[slot[r + 1]][k]);
            // xtime on planes (k = 0 is bit 7): shift left, reduce by 0x1b.
            const uint32_t x[8] = {t[1], t[2], t[3], t[4] ^ t[0], t[5] ^ t[0], t[6], t[7] ^ t[0], t[0]};
            const uint32_t* key = rk_mask + (K * 16 + 4 * c + r) * 8;
#pragma unroll
            for (int k = 0; k < 8; ++k) st[slot[r]][k] ^= x[k] ^ sum[k] ^ key[k];
        }
    }
}

// AddRoundKey of the last round (no MixColumns), after its ShiftRows.
SIB_HD void bs_add_last(uint32_t st[16][8], const uint32_t* rk_mask)
{
#pragma unroll
    for (int c = 0; c < 4; ++c)
#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
            for (int k = 0; k < 8; ++k) st[bs_slot(r, c, 10)][k] ^= rk_mask[(160 + 4 * c + r) * 8 + k];
}

SIB_HD void bs_encrypt(uint32_t st[16][8], const uint32_t* rk_mask)
{
    bs_sub_bytes(st); bs_mix_add<1>(st, rk_mask);
    bs_sub_bytes(st); bs_mix_add<2>(st, rk_mask);
    bs_sub_bytes(st); bs_mix_add<3>(st, rk_mask);
    bs_sub_bytes(st); bs_mix_add<4>(st, rk_mask);
    bs_sub_bytes(st); bs_mix_add<5>(st, rk_mask);
    bs_sub_bytes(st); bs_mix_add<6>(st, rk_mask);
    bs_sub_bytes(st); bs_mix_add<7>(st, rk_mask);
    bs_sub_bytes(st); bs_mix_add<8>(st, rk_mask);
    bs_sub_bytes(st); bs_mix_add<9>(st, rk_mask);
    bs_sub_bytes(st); bs_add_last(st, rk_mask);
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
// word w of block j.  Logical byte 4w + t sits in slot bs_slot(t, w, 10).
template <int W>
SIB_HD void bs_store_word(const uint32_t st[16][8], uint32_t out[32])
{
#pragma unroll
    for (int t = 0; t < 4; ++t)
#pragma unroll
        for (int i = 0; i < 8; ++i) out[8 * t + i] = st[bs_slot(t, W, 10)][7 - i];
    bs_transpose32(out);
}

}  // namespace sib
