"""The recorded reference results (tests/golden/ref_fixtures.npz) against the
reference build they were recorded from, and their completeness.  No GPU.

Where the reference build is present, a few recordings are re-run live and
must match bit for bit (the build is deterministic: the engine's OpenMP
loops split rows, and the softmax reduction runs nested, single-threaded).
Everywhere, every key the GPU tests read must be in the file."""
import numpy as np
import pytest

import oracle
import refsrc
import test_configs_e2e_gpu as tc
import test_engine_gpu as te
import test_sampler_gpu as ts
import test_support_ops_gpu as to


def test_every_recording_the_gpu_tests_read_exists():
    keys = set()
    for key, *_ in te.reference_runs():
        keys |= {f"{key}/{f}" for f in ("ref_tok", "top_idx", "top_val", "scale",
                                         "full_steps", "full")}
    for model in te.MODELS:
        for theta in (500000.0, 10000.0):
            keys.add(te.noise_key(model, theta))
    keys |= {ts.sampler_key(*c) for c in ts.CASES}
    keys |= {"sampler_flat", ts.argmax_key("t0")}
    keys |= {to.argmax_case_key(n, t) for n, t in to.ARGMAX_CASES}
    for key in [tc.config1_key(10000.0), tc.config1_key(500000.0), tc.CONFIG5_KEY]:
        keys |= {f"{key}/{f}" for f in ("ref_tok", "top_idx", "top_val", "scale",
                                         "full_steps", "full")}
    keys.add(tc.CONFIG5_NOISE_KEY)
    for k in sorted(keys):
        refsrc.recorded(k)
    rec = refsrc.EngineRecord.load(te.engine_key("hd64", "v1", 500000.0))
    assert rec.steps == te.STEPS["hd64"] and 0 in rec.full and rec.steps - 1 in rec.full


@pytest.mark.skipif(not oracle.has_ref_engine(), reason="needs the reference build")
def test_recordings_match_the_live_reference(tmp_path):
    paths = te.write_models(tmp_path)
    for key, model, fmt, theta, prompt, steps in te.reference_runs():
        if model != "hd128" or theta != 500000.0 or not key.startswith("engine/"):
            continue
        ref = oracle.RefEngine(paths[(model, fmt)])
        live = refsrc.run_reference(ref, prompt, steps, full_every=refsrc.FULL_EVERY)
        ref.close()
        stored = refsrc.EngineRecord.load(key)
        np.testing.assert_array_equal(live.ref_tok, stored.ref_tok)
        np.testing.assert_array_equal(live.top_val, stored.top_val)
        for s in stored.full:
            np.testing.assert_array_equal(live.full[s], stored.full[s])
    v, t, p = ts.CASES[0]
    seed, logits = ts.case_inputs(v, t, p)
    np.testing.assert_array_equal(ts.reference_draws(t, p, seed, logits),
                                  refsrc.recorded(ts.sampler_key(v, t, p)))
