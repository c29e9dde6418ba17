"""Reference results for the end-to-end parity tests: live, or recorded.

The engine and sampler parity tests compare the GPU path with the
reference's own compiled code (``oracle/_ref``: the unmodified engine behind
``Transformer::create``/``forward``, src/inference/TransformerFactory.cpp:59,
FloatTransformer.cpp:751-797, QuantizedTransformer.cpp:1014-1061, and its
``Sampler``, Sampler.cpp:133-232).  Where that library is present the tests
run it live.  Where it is not (a machine that received the tree without the
reference build), they read the same reference results from
``tests/golden/ref_fixtures.npz``, which ``tests/golden/make_ref_fixtures.py``
records by running that library on the same seeded inputs.  A test that has
neither fails; it never skips.

A recorded engine run keeps, per decode step, the reference's greedy token,
its top ``TOPK`` logits (indices and values, descending) and max|logits|, and
the full logits every ``FULL_EVERY`` steps; a live run has the full logits
at every step.  ``compare_step`` measures the GPU logits against either.
"""
from __future__ import annotations

import os

import numpy as np

import oracle

HERE = os.path.dirname(os.path.abspath(__file__))
FIXTURE = os.path.join(HERE, "golden", "ref_fixtures.npz")
TOPK = 32
FULL_EVERY = 32

_fx = None


def live() -> bool:
    """True when the reference build is present (and LEAP_REF_MODE is not
    ``recorded``, which forces the recordings, to test that path)."""
    if os.environ.get("LEAP_REF_MODE") == "recorded":
        return False
    return oracle.has_ref_engine()


def _fixtures():
    global _fx
    if _fx is None:
        if not os.path.exists(FIXTURE):
            raise RuntimeError(
                "neither the reference build (oracle/_ref) nor the recorded reference results "
                f"({FIXTURE}) are present: build the reference or regenerate the fixtures")
        with np.load(FIXTURE) as z:
            _fx = {k: z[k] for k in z.files}
    return _fx


def recorded(key: str) -> np.ndarray:
    fx = _fixtures()
    if key not in fx:
        raise KeyError(f"no recorded reference result '{key}': regenerate "
                       "tests/golden/ref_fixtures.npz with tests/golden/make_ref_fixtures.py")
    return fx[key]


class EngineRecord:
    """The reference engine's teacher-forced run: step i feeds the previous
    step's reference token (the prompt's last token first)."""

    def __init__(self, ref_tok, top_idx, top_val, scale, full_steps, full):
        self.ref_tok = np.asarray(ref_tok, np.int64)
        self.top_idx = np.asarray(top_idx, np.int64)
        self.top_val = np.asarray(top_val, np.float32)
        self.scale = np.asarray(scale, np.float32)
        self.full = {int(s): full[i] for i, s in enumerate(full_steps)}

    @property
    def steps(self) -> int:
        return int(self.ref_tok.size)

    def arrays(self, key: str) -> dict:
        steps = sorted(self.full)
        return {f"{key}/ref_tok": self.ref_tok.astype(np.int32),
                f"{key}/top_idx": self.top_idx.astype(np.int32),
                f"{key}/top_val": self.top_val,
                f"{key}/scale": self.scale,
                f"{key}/full_steps": np.asarray(steps, np.int32),
                f"{key}/full": np.stack([self.full[s] for s in steps]).astype(np.float32)}

    @classmethod
    def load(cls, key: str) -> "EngineRecord":
        return cls(recorded(f"{key}/ref_tok"), recorded(f"{key}/top_idx"),
                   recorded(f"{key}/top_val"), recorded(f"{key}/scale"),
                   recorded(f"{key}/full_steps"), recorded(f"{key}/full"))


def run_reference(ref, prompt, steps, full_every=1, topk=TOPK) -> EngineRecord:
    """Drive a reference engine (oracle.RefEngine) teacher-forced on its own
    greedy tokens and record its results."""
    for p, t in enumerate(prompt[:-1]):
        ref.forward(t, p)
    tok, pos = prompt[-1], len(prompt) - 1
    toks, idxs, vals, scales, fs, full = [], [], [], [], [], []
    for i in range(steps):
        lr = ref.forward(tok, pos)
        r_tok = ref.argmax(lr)
        order = np.argsort(-lr, kind="stable")[:topk]
        toks.append(r_tok)
        idxs.append(order)
        vals.append(lr[order])
        scales.append(float(np.abs(lr).max()))
        if i % full_every == 0 or i == steps - 1:
            fs.append(i)
            full.append(lr.copy())
        tok, pos = r_tok, pos + 1
    return EngineRecord(toks, np.stack(idxs), np.stack(vals), scales, fs, full)


def engine_reference(key: str, path: str, theta_10k: bool, prompt, steps) -> EngineRecord:
    """Live (full logits every step) when the reference build is present,
    else the recording under `key`."""
    if live():
        ref = oracle.RefEngine(path, theta_10k=theta_10k)
        try:
            return run_reference(ref, prompt, steps)
        finally:
            ref.close()
    rec = EngineRecord.load(key)
    assert rec.steps >= steps, f"recording '{key}' has {rec.steps} steps, {steps} wanted"
    return rec


def compare_step(rec: EngineRecord, i: int, le: np.ndarray, eng_tok: int):
    """(agrees, error, margin, comparable) of GPU logits `le` at step i.

    error = max|le - ref| over the full logits where the step has them, else
    over the reference's top-K entries (a lower bound of the full error).
    margin = the reference's top-2 gap.  comparable is False when the GPU's
    token lies outside the recorded top-K (only possible without the full
    logits); a disagreement there is not near a reference tie."""
    r_tok = int(rec.ref_tok[i])
    if i in rec.full:
        lr = rec.full[i]
        err = float(np.abs(le - lr).max())
        comparable = True
    else:
        idx = rec.top_idx[i]
        err = float(np.abs(le[idx] - rec.top_val[i]).max())
        comparable = eng_tok == r_tok or eng_tok in set(idx.tolist())
    margin = float(rec.top_val[i][0] - rec.top_val[i][1])
    return eng_tok == r_tok, err, margin, comparable
