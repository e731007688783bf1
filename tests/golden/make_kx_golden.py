"""Generate tests/golden/kx_vectors.json from the reference's own Monocypher.

The reference computes its session key agreement (secure_infer.cpp:449-521,
kernels/aicpu/key_agreement.aicpu:9-48) with the Monocypher copy vendored at
secure_infer/native/kernels/aicpu/monocypher/.  Build it from those sources
first, then run this script in a container that has the reference checkout:

    make -C oracle ref REFERENCE_ROOT=<path-to-secure_infer-checkout>
    python tests/golden/make_kx_golden.py

Every value in the file comes from that build; inputs are seeded.  The tests
(tests/test_kx_cpu.py) read the file and never need the build.
"""
from __future__ import annotations

import json
import random
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from oracle.kx_oracle import INFO, SALT_LABEL, Monocypher, REF_LIB  # noqa: E402

P25519 = (1 << 255) - 19


def main() -> None:
    if not REF_LIB.exists():
        raise SystemExit(f"{REF_LIB} is missing: make -C oracle ref REFERENCE_ROOT=<checkout>")
    mc = Monocypher()
    rng = random.Random(20261202)
    rb = lambda n: rng.randbytes(n)  # noqa: E731
    le = lambda v: v.to_bytes(32, "little")  # noqa: E731

    x25519 = []
    points = [rb(32) for _ in range(8)] + [le(9), le(P25519 + 1), le(P25519 - 1), b"\xff" * 32, le(0), le(1)]
    for i, u in enumerate(points):
        k = rb(32)
        x25519.append(dict(scalar=k.hex(), u=u.hex(), out=mc.x25519(k, u).hex()))
    public = []
    for _ in range(6):
        k = rb(32)
        public.append(dict(scalar=k.hex(), out=mc.x25519_public(k).hex()))
    blake = []
    for size, klen in [(1, 0), (4, 32), (16, 32), (32, 16), (64, 0), (64, 64)]:
        for mlen in (0, 1, 127, 128, 129, 300):
            key, msg = rb(klen), rb(mlen)
            blake.append(dict(size=size, key=key.hex(), msg=msg.hex(), out=mc.blake2b(msg, size, key).hex()))
    handshakes = []
    for _ in range(4):
        hs, ds, ch = rb(32), rb(32), rb(32)
        hp, dp = mc.x25519_public(hs), mc.x25519_public(ds)
        shared = mc.x25519(ds, hp)
        key = mc.blake2b(INFO + hp + dp + ch, 16, shared)
        handshakes.append(dict(host_secret=hs.hex(), device_secret=ds.hex(), challenge=ch.hex(),
                               host_public=hp.hex(), device_public=dp.hex(), shared=shared.hex(),
                               key=key.hex(), proof=mc.blake2b(ch, 32, key).hex(),
                               salt=mc.blake2b(SALT_LABEL, 4, shared).hex()))
    out = dict(source="reference Monocypher (secure_infer/native/kernels/aicpu/monocypher/monocypher.c)",
               x25519=x25519, public=public, blake2b=blake, handshakes=handshakes)
    path = Path(__file__).resolve().parent / "kx_vectors.json"
    path.write_text(json.dumps(out, indent=1) + "\n")
    print(f"wrote {path}")


if __name__ == "__main__":
    main()
