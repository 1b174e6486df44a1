"""Extracts the resampler's golden vectors from the reference's audio test
fixture (tests/fixtures/audio_golden.json of the reference tree, made by
torchaudio) into tests/golden/resample_golden.json: per case the signal
spec, the rates, the output length and every `stride`-th output sample.

Run from the repository root with the reference tree at $REF; the fixture
is copied as data, no reference code runs."""
from __future__ import annotations

import json
import os
import sys
from pathlib import Path


def main() -> None:
    if not os.environ.get("REF"):
        sys.exit("set REF to the reference tree")
    REF = Path(os.environ["REF"])
    src = json.loads((REF / "tests" / "fixtures" / "audio_golden.json").read_text())
    cases = [{"signal": e["signal"], "target": e["target"], "length": e["length"],
              "samples": e["samples"]} for e in src["resample"]]
    out = {"source": "reference tests/fixtures/audio_golden.json (resample)",
           "stride": src["stride"], "tolerance": 2e-6, "cases": cases}
    dst = Path(__file__).with_name("resample_golden.json")
    dst.write_text(json.dumps(out, indent=1) + "\n")
    print(f"wrote {dst} ({len(cases)} cases)", file=sys.stderr)


if __name__ == "__main__":
    main()
