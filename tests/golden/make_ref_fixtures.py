"""Record the reference's own results for the end-to-end parity tests.

Runs the reference build (``oracle/_ref``: the unmodified engine and its
Sampler, compiled from the reference sources by ``oracle/Makefile``) on the
same seeded inputs that ``tests/test_engine_gpu.py``,
``tests/test_sampler_gpu.py`` and ``tests/test_support_ops_gpu.py`` build,
and writes ``tests/golden/ref_fixtures.npz``.  Those tests use the
recordings only where the reference build is absent (``tests/refsrc.py``).

    python tests/golden/make_ref_fixtures.py [--part small|configs|all]

``small`` records the cases of the small models and the sampler, ``configs``
the BASELINE-shaped files of ``tests/test_configs_e2e_gpu.py`` (a 4 GB and
an 8 GB model file in a temporary directory; several minutes); other keys
already in the file are kept.  Needs the reference build
(``make -C oracle ref REF=<reference checkout>`` or
``__graft_entry__.build()``); no GPU.
"""
from __future__ import annotations

import json
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
TESTS = os.path.dirname(HERE)
ROOT = os.path.dirname(TESTS)
for p in (ROOT, TESTS):
    if p not in sys.path:
        sys.path.insert(0, p)

import oracle  # noqa: E402
import refsrc  # noqa: E402
import test_configs_e2e_gpu as tc  # noqa: E402
import test_engine_gpu as te  # noqa: E402
import test_sampler_gpu as ts  # noqa: E402
import test_support_ops_gpu as to  # noqa: E402


FIRST_AND_LAST = 1 << 30  # full logits at the first and last step only


def record_configs(out: dict) -> None:
    with tempfile.TemporaryDirectory() as d:
        p1 = tc.write_config1(d)
        prompt = te._prompt(tc.TL_PROMPT, tc.TL.vocab_size, seed=0)
        for theta in (10000.0, 500000.0):
            ref = oracle.RefEngine(p1, theta_10k=(theta == 10000.0))
            rec = refsrc.run_reference(ref, prompt, tc.TL_STEPS, full_every=FIRST_AND_LAST)
            ref.close()
            out.update(rec.arrays(tc.config1_key(theta)))
            print(tc.config1_key(theta), flush=True)
        os.remove(p1)
        p5, q5 = tc.write_config5(d)
        prompt = te._prompt(tc.L70_PROMPT, tc.L70.vocab_size, seed=0)
        ref = oracle.RefEngine(p5)
        full = refsrc.run_reference(ref, prompt, tc.L70_STEPS)
        ref.close()
        rec = refsrc.EngineRecord(full.ref_tok, full.top_idx, full.top_val, full.scale,
                                  [0, tc.L70_STEPS - 1],
                                  [full.full[0], full.full[tc.L70_STEPS - 1]])
        out.update(rec.arrays(tc.CONFIG5_KEY))
        a, w = tc.config5_noise(full, q5, prompt)
        out[tc.CONFIG5_NOISE_KEY] = np.asarray([a, w], np.float64)
        print(tc.CONFIG5_KEY, "noise", a, w, flush=True)


def main() -> None:
    import argparse
    ap = argparse.ArgumentParser()
    ap.add_argument("--part", choices=["small", "configs", "all"], default="all")
    part = ap.parse_args().part
    if not oracle.has_ref_engine():
        raise SystemExit("the reference build (oracle/_ref) is missing: build it first")
    out: dict[str, np.ndarray] = {}
    if os.path.exists(refsrc.FIXTURE):
        with np.load(refsrc.FIXTURE) as z:
            out.update({k: z[k] for k in z.files})
    if part in ("configs", "all"):
        record_configs(out)
    if part == "configs":
        save(out)
        return
    with tempfile.TemporaryDirectory() as d:
        paths = te.write_models(d)
        for key, model, fmt, theta, prompt, steps in te.reference_runs():
            ref = oracle.RefEngine(paths[(model, fmt)], theta_10k=(theta == 10000.0))
            rec = refsrc.run_reference(ref, prompt, steps, full_every=refsrc.FULL_EVERY)
            ref.close()
            out.update(rec.arrays(key))
            print(key, rec.steps, "steps", flush=True)
        for model in te.MODELS:
            for theta in (500000.0, 10000.0):
                a, w = te.noise_floor_of(paths, model, theta)
                out[te.noise_key(model, theta)] = np.asarray([a, w], np.float64)
                print(te.noise_key(model, theta), a, w, flush=True)
    for vocab, t, p in ts.CASES:
        seed, logits = ts.case_inputs(vocab, t, p)
        out[ts.sampler_key(vocab, t, p)] = ts.reference_draws(t, p, seed, logits).astype(np.int32)
    _, t, p, seed = ts.FLAT
    out["sampler_flat"] = ts.reference_draws(t, p, seed, ts.flat_inputs()).astype(np.int32)
    out[ts.argmax_key("t0")] = np.asarray(oracle.ref_argmax(ts.peaked_logits()), np.int32)
    for n, ties in to.ARGMAX_CASES:
        out[to.argmax_case_key(n, ties)] = np.asarray(
            oracle.ref_argmax(to.argmax_input(n, ties)), np.int32)
    save(out)


def save(out: dict) -> None:
    np.savez_compressed(refsrc.FIXTURE, **out)
    with open(os.path.join(HERE, "ref_fixtures.json"), "w") as f:
        json.dump({"generator": "tests/golden/make_ref_fixtures.py",
                   "reference_build": "oracle/Makefile target ref (unmodified engine, Sampler)",
                   "topk": refsrc.TOPK, "full_every": refsrc.FULL_EVERY,
                   "keys": sorted(out)}, f, indent=1)
    print("wrote", refsrc.FIXTURE, os.path.getsize(refsrc.FIXTURE), "bytes")


if __name__ == "__main__":
    main()
