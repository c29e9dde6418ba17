"""GPU: north_star's end-to-end bars on BASELINE's own model shapes, against
the reference's own engine, teacher-forced (slow: multi-GB model files).

Config 1 — TinyLlama-1.1B-shaped FP32 (v1) file: dim 2048, 22 layers,
32 q / 4 kv heads (head_dim 64), FFN 5632, vocab 32000, seq_len 2048,
weights N(0, 0.02) from seed 0, norms 1.0.  Workload as the reference's
generate loop (src/inference/main.cpp:80-107): a 32-token prompt of uniform
ids from seed 0, then 256 greedy steps (the cache grows 32 -> 288), each
step fed the reference's token.  RoPE theta 10000 (the configuration; the
reference build with that literal) and 500000 (the unmodified reference).
Bar: top-1 agreement >= 99.5 % and logits within 2e-4 of max|logits|.

Config 5, reduced — the 8-layer Llama-3-70B-shaped W8A8 (v2) file: dim
8192, 64 q / 8 kv heads (head_dim 128, kv_mul 8), FFN 28672, vocab 128256,
group 64, seq_len 8448.  The reference needs ~0.2 s per token on the host
for this file, so the 8192-token prompt of the full configuration is cut to
a 64-token prompt, then the configuration's 256 greedy steps.  Bar: within
the reference's own sensitivity (test_engine_gpu.py explains why a W8A8
forward needs one), measured against two copies of the file with one-ulp
norm perturbations in different layers: logits error <= 2x the larger of
the two, every disagreement at a reference near-tie, and top-1 agreement
no lower than the smaller of the two by more than the binomial slack of
the measured flip rate (two standard deviations over the steps, plus one
step).
The same file run as two layer-range stages [0, 4) and [4, 8) chained on
device gives bit-identical logits and tokens to the single stage.
"""
import os
import shutil

import numpy as np
import pytest
import torch

import oracle
import refsrc
from leap_b200 import ModelConfig, Transformer
from leap_b200.modelfile import write_v1, write_v2
from test_engine_gpu import V1_TOL, _prompt, _RefAsEngine, _teacher_forced

pytestmark = [pytest.mark.gpu, pytest.mark.slow]

TL = ModelConfig(2048, 5632, 22, 32, 4, 32000, 2048)
TL_PROMPT, TL_STEPS = 32, 256
L70 = ModelConfig(8192, 28672, 8, 64, 8, 128256, 8448)
L70_PROMPT, L70_STEPS = 64, 256


def config1_key(theta):
    return f"config1/{theta:g}"


CONFIG5_KEY = "config5"
CONFIG5_NOISE_KEY = "config5_noise"


def write_config1(d):
    p = os.path.join(str(d), "tinyllama_v1.bin")
    write_v1(p, TL, seed=0)
    return p


# one-ulp perturbations of the norm weights, (first float after the header,
# stride, direction): layer 0's attention norm up, layer 7's FFN norm down
L70_PERTURB = [(0, 7, np.inf), ((L70.n_layers + 7) * L70.dim, 5, -np.inf)]


def _perturbed_copy(src, dst, first, stride, direction):
    shutil.copyfile(src, dst)
    with open(dst, "r+b") as f:
        f.seek(256 + 4 * first)
        w = np.frombuffer(f.read(4 * L70.dim), np.float32).copy()
        w[::stride] = np.nextafter(w[::stride], np.float32(direction))
        f.seek(256 + 4 * first)
        f.write(w.tobytes())
    return dst


def write_config5(d):
    """(file, [perturbed copies])."""
    p = os.path.join(str(d), "l70b8_v2.bin")
    write_v2(p, L70, seed=0)
    copies = [_perturbed_copy(p, os.path.join(str(d), f"l70b8_v2_ulp{i}.bin"), *pt)
              for i, pt in enumerate(L70_PERTURB)]
    return p, copies


def config5_noise(rec, copies, prompt):
    """The perturbed copies of the file against the reference run `rec`
    (live): (lowest agreement, largest worst error)."""
    agree, worst = 1.0, 0.0
    for q in copies:
        b = oracle.RefEngine(q)
        try:
            a, w = _teacher_forced(rec, _RefAsEngine(b), prompt, L70_STEPS, check_ties=False)
        finally:
            b.close()
        agree, worst = min(agree, a), max(worst, w)
    return agree, worst


def accept_w8a8(agree, worst, floor, steps):
    f_agree, f_worst = floor
    flips = 1.0 - f_agree
    slack = max(0.01, 2.0 * np.sqrt(flips * (1.0 - flips) / steps) + 1.0 / steps)
    assert worst <= 2 * f_worst, (worst, f_worst)
    assert agree >= min(0.995, f_agree - slack), (agree, f_agree, slack)


@pytest.fixture(scope="module")
def config1_file(tmp_path_factory):
    return write_config1(tmp_path_factory.mktemp("config1"))


@pytest.fixture(scope="module")
def config5_files(tmp_path_factory):
    return write_config5(tmp_path_factory.mktemp("config5"))


@pytest.mark.parametrize("theta", [10000.0, 500000.0])
def test_config1_tinyllama_teacher_forced(cuda, config1_file, theta):
    prompt = _prompt(TL_PROMPT, TL.vocab_size, seed=0)
    rec = refsrc.engine_reference(config1_key(theta), config1_file, theta == 10000.0, prompt,
                                  TL_STEPS)
    with Transformer.create(config1_file, rope_theta=theta) as eng:
        agree, worst = _teacher_forced(rec, eng, prompt, TL_STEPS, batched_prompt=True)
    print(f"config 1 theta {theta:g}: top-1 agreement {agree:.4f}, worst {worst:.3g}")
    assert agree >= 0.995, agree
    assert worst <= V1_TOL, worst


def test_config5_reduced_w8a8_teacher_forced_and_two_stages(cuda, config5_files):
    path, perturbed = config5_files
    prompt = _prompt(L70_PROMPT, L70.vocab_size, seed=0)
    rec = refsrc.engine_reference(CONFIG5_KEY, path, False, prompt, L70_STEPS)
    if refsrc.live():
        floor = config5_noise(rec, perturbed, prompt)
    else:
        a, w = refsrc.recorded(CONFIG5_NOISE_KEY)
        floor = (float(a), float(w))
    with Transformer.create(path) as eng:
        agree, worst = _teacher_forced(rec, eng, prompt, L70_STEPS, batched_prompt=True)
    print(f"config 5 (8 layers): top-1 agreement {agree:.4f}, worst {worst:.3g}, "
          f"reference self {floor}")
    accept_w8a8(agree, worst, floor, L70_STEPS)

    # two layer-range stages on device against the single stage, bit for bit
    full = Transformer.create(path)
    s0 = Transformer.create(path, layer_range=(0, 4))
    s1 = Transformer.create(path, layer_range=(4, 8))
    try:
        for s in (full, s0, s1):
            s.bind_torch_stream()
        x = torch.empty((L70_PROMPT, L70.dim), device="cuda")
        logits = torch.empty(L70.vocab_size, device="cuda")
        tok_d = torch.empty(1, dtype=torch.int32, device="cuda")
        n = L70_PROMPT - 1
        s0.embed(prompt[:-1], x[:n])
        s0.layers(0, x[:n])
        s1.layers(0, x[:n])
        full.prefill(prompt[:-1], 0)
        tok, pos = prompt[-1], n
        for _ in range(8):
            lf = full.forward(tok, pos)
            x1 = x[:1]
            s0.embed([tok], x1)
            s0.layers(pos, x1)
            s1.layers(pos, x1)
            s1.head(x1, logits, tok_d)
            torch.cuda.synchronize()
            assert np.array_equal(logits.cpu().numpy(), lf)
            assert int(tok_d.item()) == full.last_token
            tok, pos = full.last_token, pos + 1
    finally:
        for s in (full, s0, s1):
            s.close()
