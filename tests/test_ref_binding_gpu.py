"""GPU: the reference's own engine with its attention block bound to the C ABI.

oracle/Makefile (target `binding`) builds the reference engine from its
sources with each run_layer's attention block (FloatTransformer.cpp:404-662,
QuantizedTransformer.cpp:680-923) replaced by one call of
leap_attn_decode_host through oracle/ref_binding_attn.cpp, the binding an
integrator adds to the reference.  Everything else (weights, projections,
FFN, sampling, Transformer::create/forward) is the reference's code.  That
engine must generate what the unmodified reference generates:

* FP32 (v1): the same greedy tokens, free-running from the prompt, and
  logits within 2e-4 of max|logits| (the decode attention agrees with the
  reference block to ~1e-6, so no step is near enough a tie to flip);
* W8A8 (v2): teacher-forced, the acceptance of test_engine_gpu.py (within
  the reference's own one-ulp self-sensitivity).
"""
import numpy as np
import pytest

import oracle
import refsrc
from test_engine_gpu import (MODELS, STEPS, V1_TOL, _accept, _prompt, _RefAsEngine,
                             _teacher_forced, noise_key, write_models)

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def files(tmp_path_factory):
    if not oracle.has_ref_binding():
        # built by __graft_entry__.build() wherever the reference sources are
        assert not oracle.has_ref_engine(), (
            "oracle/_ref has the reference engine but not its C-ABI binding: "
            "run `make -C oracle binding REF=<reference checkout>`")
        pytest.skip("no reference build on this machine (its sources were never available)")
    return write_models(tmp_path_factory.mktemp("binding"))


def _greedy(engine, prompt, steps):
    for p, t in enumerate(prompt[:-1]):
        engine.forward(t, p)
    tok, pos = prompt[-1], len(prompt) - 1
    toks, logits = [], []
    for _ in range(steps):
        lg = engine.forward(tok, pos)
        tok, pos = engine.argmax(lg), pos + 1
        toks.append(tok)
        logits.append(lg)
    return toks, logits


@pytest.mark.parametrize("model", ["hd64", "hd128"])
def test_fp32_engine_bound_to_the_abi_generates_the_reference_tokens(cuda, files, model):
    path = files[(model, "v1")]
    prompt = _prompt(32, MODELS[model].vocab_size)
    ref = oracle.RefEngine(path)
    bound = oracle.RefEngine(path, gpu_attention=True)
    try:
        t_ref, l_ref = _greedy(ref, prompt, STEPS[model])
        t_gpu, l_gpu = _greedy(bound, prompt, STEPS[model])
    finally:
        ref.close()
        bound.close()
    assert t_gpu == t_ref
    worst = max(float(np.abs(a - b).max() / np.abs(b).max()) for a, b in zip(l_gpu, l_ref))
    print(f"{model} v1: {len(t_ref)} greedy tokens identical, worst logits error {worst:.2e}")
    assert worst <= V1_TOL


@pytest.mark.parametrize("model", ["hd64", "hd128"])
def test_w8a8_engine_bound_to_the_abi_within_reference_sensitivity(cuda, files, model):
    path = files[(model, "v2")]
    prompt = _prompt(32, MODELS[model].vocab_size)
    ref = oracle.RefEngine(path)
    bound = oracle.RefEngine(path, gpu_attention=True)
    try:
        rec = refsrc.run_reference(ref, prompt, STEPS[model])
        agree, worst = _teacher_forced(rec, _RefAsEngine(bound), prompt, STEPS[model])
    finally:
        ref.close()
        bound.close()
    a, w = refsrc.recorded(noise_key(model, 500000.0))
    print(f"{model} v2: agreement {agree:.4f}, worst {worst:.3g} (reference self {a:.4f}, {w:.3g})")
    _accept("v2", agree, worst, (float(a), float(w)))
