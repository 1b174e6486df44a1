"""Extracts the decoding golden vectors of the reference's own fixture.

Usage: python tests/golden/make_decoding_golden.py REFERENCE_ROOT

Reads REFERENCE_ROOT/tests/fixtures/generator_golden.json (written by the
reference's tools/reference/generator_golden.py from k2-fsa's model) and
keeps what its decoding test uses (tests/decoding_test.cpp:40-66): the
decoding config, and per generation case the target frame count, the
32-step unmask schedule, the conditional input ids, audio_start and the
reference codes.  Writes tests/golden/decoding_golden.json.
"""
import json
import sys
from pathlib import Path


def main() -> None:
    if len(sys.argv) < 2:
        sys.exit("usage: make_decoding_golden.py REFERENCE_ROOT")
    root = Path(sys.argv[1])
    source = json.loads((root / "tests/fixtures/generator_golden.json").read_text())
    out = {"source": "reference tests/fixtures/generator_golden.json (decoding fields)",
           "config": source["config"], "generate": []}
    for entry in source["generate"]:
        out["generate"].append({key: entry[key] for key in (
            "text", "target", "schedule", "input_ids", "audio_start", "reference_codes")})
    path = Path(__file__).with_name("decoding_golden.json")
    path.write_text(json.dumps(out, separators=(",", ":")) + "\n")
    print(f"wrote {path} ({path.stat().st_size} bytes)")


if __name__ == "__main__":
    main()
