// Test driver for the host build of secure_infer_b200/csrc/kx.cuh: one request
// per stdin line, one hex answer per stdout line.
//   x <scalar> <u>            X25519(scalar, u)
//   p <scalar>                X25519(scalar, 9)
//   b <outlen> <key|-> <msg|->  BLAKE2b, keyed when key is given
//   d <shared> <host public> <device public> <challenge>
//                             session key, proof and salt, space separated
#include "kx.cuh"

#include <cstdio>
#include <cstring>
#include <iostream>
#include <sstream>
#include <string>
#include <vector>

static std::vector<uint8_t> unhex(const std::string& s)
{
    std::vector<uint8_t> out;
    if (s == "-") return out;
    for (size_t i = 0; i + 1 < s.size(); i += 2) out.push_back(static_cast<uint8_t>(std::stoi(s.substr(i, 2), nullptr, 16)));
    return out;
}

static void put(const uint8_t* p, size_t n)
{
    for (size_t i = 0; i < n; ++i) std::printf("%02x", p[i]);
}

int main()
{
    std::string line;
    while (std::getline(std::cin, line)) {
        std::istringstream in(line);
        std::string op;
        in >> op;
        if (op == "x") {
            std::string k, u;
            in >> k >> u;
            const auto kb = unhex(k), ub = unhex(u);
            uint8_t out[32];
            kx::x25519(out, kb.data(), ub.data());
            put(out, 32);
        } else if (op == "p") {
            std::string k;
            in >> k;
            const auto kb = unhex(k);
            uint8_t out[32];
            kx::x25519_public(out, kb.data());
            put(out, 32);
        } else if (op == "b") {
            uint32_t outlen;
            std::string key, msg;
            in >> outlen >> key >> msg;
            const auto kb = unhex(key), mb = unhex(msg);
            uint8_t out[64];
            kx::blake2b(out, outlen, kb.data(), static_cast<uint32_t>(kb.size()), mb.data(), mb.size());
            put(out, outlen);
        } else if (op == "d") {
            std::string a, b, c, d;
            in >> a >> b >> c >> d;
            const auto shared = unhex(a), hp = unhex(b), dp = unhex(c), ch = unhex(d);
            uint8_t key[16], proof[32], salt[4];
            kx::derive_key(key, shared.data(), hp.data(), dp.data(), ch.data());
            kx::derive_proof(proof, key, ch.data());
            kx::derive_salt(salt, shared.data());
            put(key, 16);
            std::printf(" ");
            put(proof, 32);
            std::printf(" ");
            put(salt, 4);
        } else {
            return 2;
        }
        std::printf("\n");
    }
    return 0;
}
