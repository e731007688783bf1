"""The bitsliced AES-128 counter-mode core (secure_infer_b200/csrc/
bitsliced_aes.cuh, host build through tests/bs_driver.cpp) against the
oracle's FIPS-197 AES, and its S-box circuit against the FIPS-197 S-box."""
from __future__ import annotations

import os
import shutil
import struct
import subprocess
import sys

import pytest

from conftest import ROOT, det_bytes
from oracle import gcm as orc


def test_sbox_circuit_generator_checks_all_inputs():
    """The generator refuses to write a circuit that disagrees with the S-box
    anywhere; the committed header is what it writes."""
    gen = ROOT / "secure_infer_b200" / "csrc" / "gen_bitsliced_sbox.py"
    sys.path.insert(0, str(gen.parent))
    import gen_bitsliced_sbox as g
    g.check()
    assert (gen.parent / "bitsliced_sbox.cuh").read_text() == g.emit()


@pytest.fixture(scope="module")
def driver(tmp_path_factory):
    cxx = shutil.which("g++")
    if cxx is None:
        pytest.skip("g++ not available")
    exe = tmp_path_factory.mktemp("bs") / "bs_driver"
    subprocess.run([cxx, "-O1", "-std=c++17", "-I", str(ROOT / "secure_infer_b200" / "csrc"),
                    str(ROOT / "tests" / "bs_driver.cpp"), "-o", str(exe)], check=True)
    return exe


def test_bitsliced_groups_match_oracle_aes(driver):
    """32 counter blocks per group, groups 0 (holds E_K(J0) at v = 1), 1, a
    group above 2^16 and the last group before the 32-bit counter wraps, for
    several keys and IVs."""
    import numpy as np
    cases, expect = [], []
    for t in range(6):
        key = det_bytes(f"bs-key{t}", 16)
        rk = np.zeros(176, np.uint8)
        orc.lib().orc_aes128_expand(orc._ptr(orc._buf(key)), orc._ptr(rk))
        nonce = det_bytes(f"bs-iv{t}", 12)
        iv = struct.unpack(">III", nonce)
        for g in (0, 1, 77 + t, 70000 + t, (1 << 27) - 1):
            cases.append(f"{rk.tobytes().hex()} {iv[0]:08x} {iv[1]:08x} {iv[2]:08x} {g}")
            expect.append(b"".join(orc.aes_block(key, nonce + struct.pack(">I", 32 * g + j)) for j in range(32)))
    out = subprocess.run([str(driver)], input="\n".join(cases) + "\n", capture_output=True, text=True, check=True)
    got = [bytes.fromhex(line) for line in out.stdout.split()]
    assert len(got) == len(expect)
    for i, (a, b) in enumerate(zip(got, expect)):
        assert a == b, i
