"""Generate the oracle golden fixtures of the large configs (CPU only).

The CPU oracle (``oracle/``, the C++ restatement of the reference's token
loop) is too slow to run inside a GPU test at these sizes, so it runs once
here and its answers are committed as small compressed fixtures that the
``-m gpu`` tests compare against:

  s3_4096.npz     Qwen2.5-1.5B, a 4096-id prompt (seed 1238 prompt stream),
                  32 greedy steps, f32 KV cache (long-context config)
  q14b_512.npz    Qwen2.5-14B (untied lm_head), a 512-id prompt (seed 1234),
                  16 greedy steps
  batch_512.npz   Qwen2.5-1.5B, 4 of the batched config's 64 sequences
                  (prompt seeds 5000 + b for b in 0, 21, 42, 63), 512-id
                  prompts, 128 greedy steps each

Each fixture holds the greedy ids, the oracle's top-1/top-2 logit gap at
every step (the near-tie rule of the parity tests), and logits at fixed
indices: the 256 largest entries plus 4096 seeded random indices, of the
prefill's last-token logits and of the final step's logits.

Weights are the seeded synthetic tables of ``myos.synth`` (the BASELINE
recipe), so the fixtures hold no model bytes. Run from the repository root:

    python tests/golden/make_goldens.py s3|q14b|batch [--threads N]
"""
from __future__ import annotations

import argparse
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
PKG = os.path.join(REPO, "an-operating-system-for-ai-models-and-tensor-inference_b200")
for p in (REPO, PKG, os.path.join(REPO, "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)

SEED = 1234
N_TOP, N_RAND = 256, 4096

# name -> (model, prompt seeds, n_prompt, n_gen)
CONFIGS = {
    "s3": ("1.5b", [SEED + 4], 4096, 32),
    "q14b": ("14b", [SEED], 512, 16),
    "batch": ("1.5b", [5000 + b for b in (0, 21, 42, 63)], 512, 128),
}
FILES = {"s3": "s3_4096.npz", "q14b": "q14b_512.npz", "batch": "batch_512.npz"}


def sample_index(vocab: int, logits: np.ndarray, seed: int) -> np.ndarray:
    """The N_TOP largest entries (stable order) plus N_RAND seeded indices."""
    top = np.argsort(-logits, kind="stable")[:N_TOP]
    rnd = np.random.default_rng(seed).choice(vocab, N_RAND, replace=False)
    return np.unique(np.concatenate([top, rnd])).astype(np.int64)


def run(name: str, threads: int) -> str:
    from myos import synth
    from oracle import oracle as orc

    import ref_fixtures as rf

    model, seeds, n_prompt, n_gen = CONFIGS[name]
    shape = synth.shape_qwen25_1_5b() if model == "1.5b" else synth.shape_qwen25_14b()
    orc.build()
    orc.set_threads(threads)
    t0 = time.time()
    table = synth.weights(shape, SEED, threads)
    wm = rf.load_into_oracle(orc, table)
    print(f"[{name}] weights ready in {time.time() - t0:.1f}s", flush=True)
    out = {"n_prompt": np.int64(n_prompt), "n_gen": np.int64(n_gen),
           "prompt_seeds": np.asarray(seeds, np.int64), "weight_seed": np.int64(SEED)}
    ids_all, gap_all, pre_idx, pre_val, fin_idx, fin_val = [], [], [], [], [], []
    for s in seeds:
        prompt = synth.prompt_ids(s, n_prompt, shape["vocab"])
        md = orc.Model(rf.oracle_shape(orc, shape), n_prompt + n_gen)
        t1 = time.time()
        assert md.prefill(wm, prompt) == 0
        pre = md.logits()
        t2 = time.time()
        st, ids, gap, _ = md.greedy_decode(wm, n_gen)
        assert st == 0
        fin = md.logits()
        t3 = time.time()
        print(f"[{name}] seed {s}: prefill {t2 - t1:.1f}s, {n_gen} steps {t3 - t2:.1f}s, "
              f"ids[:8] {ids[:8].tolist()}", flush=True)
        pi = sample_index(shape["vocab"], pre, s)
        fi = sample_index(shape["vocab"], fin, s + 1)
        ids_all.append(ids)
        gap_all.append(gap)
        pre_idx.append(pi)
        pre_val.append(pre[pi])
        fin_idx.append(fi)
        fin_val.append(fin[fi])
        del md
    out["ids"] = np.stack(ids_all).astype(np.uint32)
    out["gap"] = np.stack(gap_all).astype(np.float32)
    # ragged index sets: stored flat with offsets
    for key, idx, val in (("prefill", pre_idx, pre_val), ("final", fin_idx, fin_val)):
        out[key + "_off"] = np.cumsum([0] + [len(i) for i in idx]).astype(np.int64)
        out[key + "_idx"] = np.concatenate(idx).astype(np.int64)
        out[key + "_val"] = np.concatenate(val).astype(np.float32)
    path = os.path.join(HERE, FILES[name])
    np.savez_compressed(path, **out)
    print(f"[{name}] wrote {path} in {time.time() - t0:.1f}s", flush=True)
    return path


def load(name: str) -> dict:
    """Fixture arrays by key (used by the GPU tests)."""
    with np.load(os.path.join(HERE, FILES[name])) as z:
        return {k: z[k] for k in z.files}


def sampled(g: dict, key: str, i: int):
    """(indices, values) of sequence i's sampled `key` logits ('prefill'/'final')."""
    off = g[key + "_off"]
    return g[key + "_idx"][off[i]:off[i + 1]], g[key + "_val"][off[i]:off[i + 1]]


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("config", choices=sorted(CONFIGS))
    ap.add_argument("--threads", type=int, default=os.cpu_count() or 8)
    a = ap.parse_args()
    run(a.config, a.threads)
