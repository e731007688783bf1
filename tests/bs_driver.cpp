// CPU driver for secure_infer_b200/csrc/bitsliced_aes.cuh (test infrastructure).
// Each input line: 176 round-key bytes (hex), three IV words (hex), a counter
// group g (decimal).  Output line: the 32 blocks E_K(IV || BE32(32 g + j)),
// j = 0..31, as 512 bytes of hex.
#include <cstdio>
#include <cstdint>
#include <iostream>
#include <string>

#include "bitsliced_aes.cuh"

int main()
{
    std::string rk_hex;
    uint32_t iv[3];
    uint32_t g;
    while (std::cin >> rk_hex >> std::hex >> iv[0] >> iv[1] >> iv[2] >> std::dec >> g) {
        uint8_t rk[176];
        for (int i = 0; i < 176; ++i) rk[i] = static_cast<uint8_t>(std::stoul(rk_hex.substr(2 * i, 2), nullptr, 16));
        static uint32_t mask[1408];
        sib::bs_round_key_masks(rk, mask);
        uint32_t st[16][8];
        sib::bs_load_group(st, iv, g, mask);
        sib::bs_encrypt(st, mask);
        uint32_t words[4][32];
        sib::bs_store_word<0>(st, words[0]);
        sib::bs_store_word<1>(st, words[1]);
        sib::bs_store_word<2>(st, words[2]);
        sib::bs_store_word<3>(st, words[3]);
        for (int j = 0; j < 32; ++j)
            for (int w = 0; w < 4; ++w)
                for (int t = 0; t < 4; ++t) std::printf("%02x", (words[w][j] >> (8 * t)) & 0xffu);
        std::printf("\n");
    }
    return 0;
}
