"""Writes tests/golden/generation_golden.npz: full-shape 32-step CFG
generations of the CPU oracle (oracle/oracle.cpp, the restatement of the
reference's Generator::Generate, generator.cpp:486-543) on the default
28-layer, vocabulary-151936 model with random-init weights of seed 0.

Cases (each with the reference's own noise stream, std::mt19937_64 of its
seed as in decoding.cpp:64-68,84-85):
  c1        BASELINE config 1: 40 text ids U[0, 151935] (numpy seed 0),
            100 masked frames, generation seed 0;
  c2        BASELINE config 2: 120 text ids U[0, 151935] (numpy seed 1),
            250 masked frames, generation seed 1;
  c3        BASELINE config 3: 180 text ids and 150 frames of reference codes
            U[0, 1023] (numpy seed 2), 375 masked frames, generation seed 2;
  c4_<i>    six utterances of the BASELINE config-4 set (64 utterances,
            numpy seed 4: F ~ U[50, 750], text = round(0.4 F), half with
            125-250 reference frames), the six with the fewest packed rows
            (one of them with reference codes); generation seed 1000 + i.
Per case it stores the conditional ids, audio_start, the frame count, the
seed and the oracle's codes and unmasked_at ([8][F] int32 each).  The GPU
test (tests/test_gpu_fullshape.py) generates the same inputs and compares.

For configs 1, 2 and 3 it also stores the oracle's trajectory: per step the
ids the forward pass saw and the scoring's predictions and confidences, so
the GPU can be compared step by step on identical inputs.

The bar the comparisons are held to comes from the oracle itself, run
with its linear layers' float32 sums in the opposite order
(oc_set_accumulation_order(1)): an equally valid restatement of the
reference's float32 accumulation, whose order hipBLAS leaves unspecified.
Stored per case: that variant's agreement with the oracle (codes and
unmasked_at of the free-running generation) and, for config 1, its
per-step prediction agreement on the oracle's trajectory.

Usage: python tests/golden/make_generation_golden.py [--threads N] [--only NAME ...]
(about 50 minutes on 8 cores for every case; --only recomputes the named
cases and keeps the others already in the file).
"""
from __future__ import annotations

import argparse
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

VOCAB = 151936


def cases():
    from omnivoice_b200 import ConditionalInput
    out = []
    rng = np.random.default_rng(0)
    inp = ConditionalInput.build(rng.integers(0, VOCAB, size=40).tolist(), None, 100)
    out.append(("c1", inp, 0))
    rng = np.random.default_rng(1)
    inp = ConditionalInput.build(rng.integers(0, VOCAB, size=120).tolist(), None, 250)
    out.append(("c2", inp, 1))
    rng = np.random.default_rng(2)
    text = rng.integers(0, VOCAB, size=180).tolist()
    ref = rng.integers(0, 1024, size=(8, 150)).astype(np.int32)
    out.append(("c3", ConditionalInput.build(text, ref, 375), 2))
    # The config-4 set, drawn exactly as bench.py's batched_set().
    rng = np.random.default_rng(4)
    frames = rng.integers(50, 751, size=64)
    with_ref = set(rng.permutation(64)[:32].tolist())
    specs = []
    for i, f in enumerate(frames):
        ref = int(rng.integers(125, 251)) if i in with_ref else 0
        specs.append((int(round(0.4 * f)), ref, int(f)))
    inputs = []
    for text, ref, target in specs:
        ids = rng.integers(0, VOCAB, size=text).tolist()
        codes = rng.integers(0, 1024, size=(8, ref)).astype(np.int32) if ref else None
        inputs.append(ConditionalInput.build(ids, codes, target))
    rows = sorted(range(64), key=lambda i: specs[i][0] + specs[i][1] + 2 * specs[i][2])
    chosen = rows[:6]
    for i in chosen:
        out.append((f"c4_{i}", inputs[i], 1000 + i))
    return out


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--threads", type=int, default=0)
    parser.add_argument("--only", nargs="*", default=None)
    args = parser.parse_args()
    from oracle import binding
    import os
    binding.oracle().oc_set_threads(args.threads or os.cpu_count() or 1)
    model = binding.OracleModel(binding.config(), 0)
    lib = binding.oracle()
    path = Path(__file__).with_name("generation_golden.npz")
    arrays = {}
    if args.only is not None and path.exists():
        arrays = {k: v for k, v in np.load(path).items() if k != "names"}
    for name, inp, seed in cases():
        if args.only is not None and name not in args.only:
            continue
        t0 = time.time()
        lib.oc_set_accumulation_order(0)
        codes, when, step_ids, step_pred, step_conf = model.generate_traced(
            inp.ids, inp.audio_start, inp.target_frames, seed=seed)
        arrays[f"{name}_ids"] = inp.ids.astype(np.int32)
        arrays[f"{name}_meta"] = np.array([inp.audio_start, inp.target_frames, seed], np.int64)
        arrays[f"{name}_codes"] = codes
        arrays[f"{name}_unmasked_at"] = when
        # The reversed-sum restatement, free running.
        lib.oc_set_accumulation_order(1)
        v_codes, v_when = model.generate(inp.ids, inp.audio_start, inp.target_frames, seed=seed)
        agreement = [float((v_codes == codes).mean()), float((v_when == when).mean())]
        if name in ("c1", "c2", "c3"):
            arrays[f"{name}_step_ids"] = step_ids
            arrays[f"{name}_step_prediction"] = step_pred
            arrays[f"{name}_step_confidence"] = step_conf
            # ... and step by step on the oracle's own trajectory.
            same = total = 0
            for step in range(step_ids.shape[0]):
                masked = step_ids[step][:, inp.length - inp.target_frames:] == 1024
                if not masked.any():
                    continue
                logits = model.forward(step_ids[step], inp.audio_start, inp.target_frames)
                pred, _ = binding.score(logits, inp.target_frames)
                same += int((pred == step_pred[step])[masked].sum())
                total += int(masked.sum())
            agreement.append(same / total)
        arrays[f"{name}_variant_agreement"] = np.array(agreement, np.float64)
        lib.oc_set_accumulation_order(0)
        print(f"{name}: L={inp.length} F={inp.target_frames} seed={seed}, reversed-sum "
              f"restatement agrees {agreement} ({time.time() - t0:.0f} s)", flush=True)
    model.close()
    np.savez_compressed(path, names=np.array([n for n, _, _ in cases()]), **arrays)
    print(f"wrote {path} ({path.stat().st_size} bytes)")


if __name__ == "__main__":
    main()
