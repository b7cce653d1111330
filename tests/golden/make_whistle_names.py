"""Copies the reference's golden tensor map of whistle.cact
(internal/cact/testdata/whistle_names.txt, 681 records: index, name, shape,
transform, safetensors source[layer]) into tests/golden/, after checking
that every record line parses. Run once, in a checkout of the reference:

    python tests/golden/make_whistle_names.py <reference checkout>
"""

from __future__ import annotations

import sys
from pathlib import Path


def main(ref: str) -> None:
    src = Path(ref) / "internal" / "cact" / "testdata" / "whistle_names.txt"
    text = src.read_text()
    rows = [ln for ln in text.splitlines() if ln.strip() and not ln.startswith("#")]
    for k, ln in enumerate(rows):
        f = ln.split()
        assert len(f) == 5 and int(f[0]) == k and f[2].startswith("(") and f[2].endswith(")"), ln
    out = Path(__file__).resolve().parent / "whistle_names.txt"
    out.write_text(text)
    print(f"{out}: {len(rows)} records")


if __name__ == "__main__":
    main(sys.argv[1])
