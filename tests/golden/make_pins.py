"""Regenerate tests/golden/reference_pins.json from the reference's own test sources, read as text.

The reference (gladia-research-group/perseus) is Rust and cannot be built in this image, so its known-answer tests
cannot run here. Their constants are parsed out of the test files instead and committed, so the oracle's pin tests
(tests/test_oracle_pins.py) run on any machine without the reference tree:

- crates/pc-core/tests/kskb_frozen.rs: the frozen u64 key-switching-key expander (KSKB lane) seed and the pinned
  (p, a[0], a[1], a[n-1], FNV-1a of the row) tuples of digits 0 / 3 / 6 at n = 2^16;
- crates/pc-core/src/params/nbtheory.rs (tests): prime test / prime search / minimal 2N-th root answers.

Usage: python tests/golden/make_pins.py <reference root>
"""
import json
import os
import re
import sys


def _ints(s):
    return [int(x.replace("_", ""), 0) for x in re.findall(r"0x[0-9a-fA-F_]+|\d[\d_]*", s)]


def main(root):
    kf = open(os.path.join(root, "crates/pc-core/tests/kskb_frozen.rs")).read()
    seed = _ints(re.search(r"const SEED: KskSeed = KskSeed\(\[(.*?)\]\)", kf, re.S).group(1))
    digits = [int(d) for d in re.findall(r"\((\d+)u?3?2?, (?:primes|\*primes)", kf)]
    body = re.search(r"const PINNED:.*?= \[(.*?)\];", kf, re.S).group(1)
    tuples = [_ints(t) for t in re.findall(r"\(([^()]*)\)", body)]
    nb = open(os.path.join(root, "crates/pc-core/src/params/nbtheory.rs")).read()
    tests = nb[nb.index("fn primes_and_roots"):]
    prime = int(re.search(r"assert!\(is_prime\((\d+)\)\)", tests).group(1))
    pseudo = int(re.search(r"assert!\(!is_prime\((\d+)\)\);\s*//", tests).group(1))
    prev = int(re.search(r"assert_eq!\(q, (\d+)\)", tests).group(1))
    root_ans = re.search(r"assert_eq!\(root_of_unity\(m, (\d+)\)\.unwrap\(\), (\d+)\)", tests)
    out = {
        "source": "parsed from the reference test files by tests/golden/make_pins.py",
        "kskb_frozen": {
            "file": "crates/pc-core/tests/kskb_frozen.rs",
            "logn": 16,
            "seed": seed,
            "digits": digits,
            "pinned": tuples,
        },
        "nbtheory": {
            "file": "crates/pc-core/src/params/nbtheory.rs",
            "prime": prime,
            "composite": prime * 3,
            "strong_pseudoprime": pseudo,
            "m": 1 << 17,
            "previous_of_first_28": prev,
            "root_prime": int(root_ans.group(1)),
            "root": int(root_ans.group(2)),
        },
    }
    assert len(seed) == 8 and len(tuples) == 3 and len(digits) == 3, (seed, tuples, digits)
    dst = os.path.join(os.path.dirname(os.path.abspath(__file__)), "reference_pins.json")
    with open(dst, "w") as f:
        json.dump(out, f, indent=1)
    print("wrote", dst)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_pins.py <reference root>")
    main(sys.argv[1])
