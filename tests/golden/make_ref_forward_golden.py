"""Produces tests/golden/ref_forward_tiny_q6k.npz by running the reference's own CUDA forward
(src/model/qwen3.cu, rebuilt unmodified for sm_100a as oracle/_ref/ref_model) on the seeded
tiny-q6k synthetic model: a 24-token prompt, then 16 teacher-forced decode steps, recording the
fp32 logits and greedy id of every step. Needs a GPU (run it on the B200 box):

    python tests/golden/make_ref_forward_golden.py [OUT.npz]

The CPU oracle's full forward is pinned against this file in tests/test_oracle_pins.py.
"""
import os
import subprocess
import sys
import tempfile

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, ROOT)
import oracle as orc  # noqa: E402
from __graft_entry__ import _load_pkg  # noqa: E402

MODEL_CONFIG, MODEL_SEED = "tiny-q6k", 21
N_PROMPT, N_STEPS = 24, 16


def fixture_tokens():
    rng = np.random.default_rng(424242)
    prompt = rng.integers(0, 2048, N_PROMPT).tolist()
    teacher = rng.integers(0, 2048, N_STEPS).tolist()
    return prompt, teacher


def run_reference(model_path, prompt, teacher, steps, max_ctx, out_path, logits=True, binary=None):
    cmd = [binary or orc.REF_MODEL, model_path, out_path, "--tokens", ",".join(map(str, prompt)), "--steps", str(steps),
           "--max-ctx", str(max_ctx)]
    if teacher:
        cmd += ["--teacher", ",".join(map(str, teacher))]
    if not logits:
        cmd.append("--no-logits")
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=1800)
    if r.returncode != 0:
        raise RuntimeError(f"ref_model failed ({r.returncode}): {r.stderr[-2000:]}")
    return orc.read_ref_dump(out_path), r.stdout


def main():
    out = sys.argv[1] if len(sys.argv) > 1 else os.path.join(os.path.dirname(os.path.abspath(__file__)),
                                                             "ref_forward_tiny_q6k.npz")
    fb = _load_pkg()
    prompt, teacher = fixture_tokens()
    with tempfile.TemporaryDirectory() as d:
        p = os.path.join(d, "m.gguf")
        fb.synth_write(p, MODEL_CONFIG, seed=MODEL_SEED)
        (V, n_prompt, ids, logits), _ = run_reference(p, prompt, teacher, N_STEPS, 256, os.path.join(d, "dump.bin"))
    np.savez(out, prompt=np.array(prompt, np.int32), teacher=np.array(teacher, np.int32), ids=ids, logits=logits,
             config=MODEL_CONFIG, seed=MODEL_SEED)
    print("wrote", out, "logits std", float(logits.std()))


if __name__ == "__main__":
    main()
