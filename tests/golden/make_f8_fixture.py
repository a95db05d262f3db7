"""Writes f8_tables.json: the reference's own conversion tables, read as text from its sources.

  F8E4_TO_F32      furiosa-opt-std/src/float/f8e4.rs (the 256-entry f8e4m3 -> f32 table)
  F4E2M1_TO_F8E4   furiosa-opt-std/src/scalar.rs     (the 16-entry e2m1 -> f8e4m3 table)

Run once where the reference checkout exists: python tests/golden/make_f8_fixture.py <reference root>.
The CPU tests compare the oracle's f8 decode and f4 lookup with these tables entry by entry.
"""
import json
import os
import re
import sys


def table(text: str, name: str):
    body = re.search(name + r"[^=]*=\s*&?\[(.*?)\];", text, re.S).group(1)
    return [int(x, 16) for x in re.findall(r"0x[0-9a-fA-F]+", body)]


def main(root: str):
    std = os.path.join(root, "furiosa-opt-std", "src")
    e4 = table(open(os.path.join(std, "float", "f8e4.rs")).read(), "const F8E4_TO_F32")
    f4 = table(open(os.path.join(std, "scalar.rs")).read(), "const F4E2M1_TO_F8E4")
    assert len(e4) == 256 and len(f4) == 16
    out = os.path.join(os.path.dirname(os.path.abspath(__file__)), "f8_tables.json")
    with open(out, "w") as fh:
        json.dump({"source": {"F8E4_TO_F32": "furiosa-opt-std/src/float/f8e4.rs",
                              "F4E2M1_TO_F8E4": "furiosa-opt-std/src/scalar.rs"},
                   "F8E4_TO_F32": e4, "F4E2M1_TO_F8E4": f4}, fh)
    print(out)


if __name__ == "__main__":
    main(sys.argv[1])
