"""The myos CLI end to end on the GPU, against the reference CLI's own
expectations (crates/runtime/tests/weights_cli.rs) and the engine API."""
import json
import os
import struct
import subprocess

import numpy as np
import pytest

import myos
from myos import synth

pytestmark = pytest.mark.gpu

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BIN = os.path.join(REPO, "an-operating-system-for-ai-models-and-tensor-inference_b200", "lib", "myos")


def run(args, cwd, env=None, timeout=600):
    e = dict(os.environ)
    e.pop("MYOS_WEIGHTS", None)
    e.update(env or {})
    p = subprocess.run([BIN] + args, cwd=cwd, env=e, capture_output=True, text=True,
                       timeout=timeout)
    return p.returncode, p.stdout, p.stderr


def assert_bf16_fingerprint(js):
    for frag in ['"quant_or_dtype": "bf16"', '"acc_path": "bf16_w_fp32_acc"',
                 '"deterministic": true', '"model_sha256": null', '"seed": null',
                 '"scenario_id": "S1"', '"threads": 8', '"gemv_pack": false', '"batch": 1',
                 '"device": "cuda:0"']:
        assert frag in js, (frag, js)


def test_default_smoke_is_the_cycle(tmp_path):
    code, out, err = run([], tmp_path)
    assert (code, err) == (0, "")
    assert out == "MyOS Phase1 smoke decode (prompt=0): [1, 2, 3, 0]\n"
    assert not (tmp_path / "runs").exists()
    code, out, _ = run(["--steps", "2"], tmp_path)
    assert out == "MyOS Phase1 smoke decode (prompt=0): [1, 2]\n"


def test_block_fixture_tokens_and_fingerprint(tmp_path):
    code, out, err = run(["--block-fixture"], tmp_path)
    assert (code, err) == (0, "")
    assert out == "MyOS Phase1 block fixture (prompt=0): [1, 1, 1, 1]\n"
    js = (tmp_path / "runs/s1-block-fixture/run_fingerprint.json").read_text()
    assert_bf16_fingerprint(js)
    d = json.loads(js)
    assert d["layout"] == "block-fixture" and d["model_id"] is None and d["fmt"] == "in-process"
    assert (d["n_gen"], d["n_ctx"], d["n_prompt"], d["commit"]) == (4, 5, 1, None)
    assert not (tmp_path / "runs/s1-block-fixture/token_ids.txt").exists()
    # twice: the same tokens; --fingerprint-dir moves the artefacts
    code, out2, _ = run(["--block-fixture"], tmp_path)
    assert out2 == out
    code, out, err = run(["--block-fixture", "--steps", "2", "--fingerprint-dir", "fp"], tmp_path)
    assert out == "MyOS Phase1 block fixture (prompt=0): [1, 1]\n"
    d = json.loads((tmp_path / "fp/run_fingerprint.json").read_text())
    assert (d["n_gen"], d["n_ctx"]) == (2, 3)
    ref = tmp_path / "ref.txt"
    ref.write_text("1 1 1 1\n")
    _, out, _ = run(["--block-fixture", "--ref-ids", str(ref)], tmp_path)
    assert out.endswith("CORRECT: PASS\n")
    ref.write_text("1 2 1 1\n")
    code, out, _ = run(["--block-fixture", "--ref-ids", str(ref)], tmp_path)
    assert code == 0 and out.endswith("CORRECT: FAIL first_diff@1: got=1 ref=2\n")


def _safetensors(path, entries):
    header, blobs, off = {}, [], 0
    for name, dtype, shape, data in entries:
        header[name] = {"dtype": dtype, "shape": shape, "data_offsets": [off, off + len(data)]}
        off += len(data)
        blobs.append(data)
    hb = json.dumps(header).encode()
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hb)) + hb + b"".join(blobs))


def test_weight_errors_exit_1_without_artefacts(tmp_path):
    tiny = tmp_path / "tiny.safetensors"
    _safetensors(tiny, [("w", "F32", [1], struct.pack("<f", 1.0)),
                        ("bias", "F32", [], struct.pack("<f", 0.5))])
    code, out, err = run(["--weights", str(tiny)], tmp_path)
    assert code == 1 and "MyOS weights" in err and "tensor not found" in err
    assert "smoke decode" not in out and "weights decode" not in out
    # the environment selects the file; the flag wins over it
    code, out, err = run([], tmp_path, env={"MYOS_WEIGHTS": str(tiny)})
    assert code == 1 and str(tiny) in err and "smoke decode" not in out
    missing = tmp_path / "absent.safetensors"
    code, out, err = run(["--weights", str(tiny)], tmp_path, env={"MYOS_WEIGHTS": str(missing)})
    assert code == 1 and str(tiny) in err and str(missing) not in err
    code, out, err = run(["--weights", str(missing)], tmp_path)
    assert code == 1 and "MyOS weights" in err
    garbage = tmp_path / "garbage.safetensors"
    garbage.write_bytes(b"not-a-safetensors-file!!!!")
    code, out, err = run(["--weights", str(garbage)], tmp_path)
    assert code == 1 and "could not be parsed" in err
    # the miniature block is not the 1.5B layout
    import ref_fixtures as rf
    _, t = rf.block_fixture()
    _safetensors(tmp_path / "mini.safetensors",
                 [(k, "BF16", list(s), b.tobytes()) for k, (s, b) in t.items()])
    code, out, err = run(["--weights", str(tmp_path / "mini.safetensors")], tmp_path)
    assert code == 1 and "tensor shape does not match the layout" in err
    assert "[1, 1, 1, 1]" not in out
    # bad weights also stop the block fixture
    code, out, err = run(["--weights", str(garbage), "--block-fixture"], tmp_path)
    assert code == 1 and "MyOS weights" in err and "block fixture" not in out
    assert not (tmp_path / "runs").exists()


@pytest.fixture(scope="module")
def s1_file(tmp_path_factory):
    shape = synth.shape_qwen25_1_5b()
    table = synth.weights(shape, 1234)
    path = tmp_path_factory.mktemp("w") / "qwen25_1_5b_seed1234.safetensors"
    synth.write_safetensors(str(path), table)
    return shape, table, str(path)


@pytest.mark.slow
def test_weights_decode_matches_engine_and_writes_artefacts(tmp_path, s1_file):
    shape, table, path = s1_file
    prompt = synth.prompt_ids(1234, 16, shape["vocab"])
    steps = 8
    e = myos.Engine(shape, len(prompt) + steps)
    e.load_table(table)
    e.prefill(prompt, want_logits=False)
    want = e.greedy_decode(steps).tolist()
    e.close()
    pfile = tmp_path / "prompt.txt"
    pfile.write_text(" ".join(map(str, prompt.tolist())) + "\n")
    rfile = tmp_path / "ref.txt"
    rfile.write_text(" ".join(map(str, want)) + "\n")
    code, out, err = run(["--weights", path, "--prompt-ids", str(pfile), "--ref-ids", str(rfile),
                          "--steps", str(steps), "--fingerprint-dir", "run"], tmp_path)
    assert code == 0, err
    assert out == (f"MyOS Phase1 weights decode (prompt={prompt[0]}, steps={steps}): "
                   f"[{', '.join(map(str, want))}]\nCORRECT: PASS\n")
    assert (tmp_path / "run/token_ids.txt").read_text() == " ".join(map(str, want)) + "\n"
    fp = json.loads((tmp_path / "run/run_fingerprint.json").read_text())
    assert fp["model_id"] == "Qwen/Qwen2.5-1.5B-Instruct" and fp["layout"] == "qwen25_1_5b"
    assert (fp["n_prompt"], fp["n_gen"], fp["n_ctx"]) == (16, steps, 16 + steps)
    m = json.loads((tmp_path / "run/metrics.json").read_text())
    assert m["correct"] is True and (m["n_prompt"], m["n_gen"]) == (16, steps)
    assert m["T_decode_tok_s"] == pytest.approx(steps / m["t_decode_s"])
    assert m["L_TPOT_ms"] == pytest.approx(m["t_decode_s"] * 1000 / steps)
    # arena: one warm-up and two scored children, medians, CORRECT and DET
    code, out, err = run(["--arena-s1", "--weights", path, "--prompt-ids", str(pfile),
                          "--ref-ids", str(rfile), "--steps", str(steps), "--warmup", "1",
                          "--repeats", "2", "--fingerprint-dir", "arena",
                          "--cost-card", "card.md"], tmp_path, timeout=900)
    assert code == 0, err
    assert out.startswith("ARENA S1 threads=8 W=1 R=2 CORRECT=PASS DET=PASS")
    assert (tmp_path / "card.md").exists() and (tmp_path / "arena/score-2/metrics.json").exists()
