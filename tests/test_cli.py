"""The myos CLI's argument rules and exit codes (crates/runtime/src/main.rs:229-382,
crates/runtime/tests/weights_cli.rs): usage errors exit 2 before any device
work, so these run without a GPU."""
import os
import subprocess

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(REPO, "an-operating-system-for-ai-models-and-tensor-inference_b200")
BIN = os.path.join(PKG, "lib", "myos")
USAGE = ("usage: myos [--weights PATH] [--block-fixture] [--steps N] [--threads N] "
         "[--fingerprint-dir DIR] [--prompt-ids PATH] [--ref-ids PATH] [--arena-s1] "
         "[--warmup N] [--repeats N] [--cost-card PATH]")


@pytest.fixture(scope="module", autouse=True)
def built():
    import build as pkg_build

    pkg_build.build()
    assert os.path.exists(BIN)


def run(args, cwd, env=None):
    e = dict(os.environ)
    e.pop("MYOS_WEIGHTS", None)
    e.update(env or {})
    p = subprocess.run([BIN] + args, cwd=cwd, env=e, capture_output=True, text=True, timeout=60)
    return p.returncode, p.stdout, p.stderr


@pytest.mark.parametrize("args,msg", [
    (["--bogus"], "unknown argument `--bogus`"),
    (["--steps", "0"], "--steps needs a positive integer, got `0`"),
    (["--steps=x"], "--steps needs a positive integer, got `x`"),
    (["--steps"], "--steps needs a positive integer"),
    (["--weights"], "--weights needs a path"),
    (["--weights="], "--weights needs a path"),
    (["--threads", "0"], "--threads needs an integer from 1 to 64, got `0`"),
    (["--threads", "65"], "--threads needs an integer from 1 to 64, got `65`"),
    (["--prompt-ids", "p.txt"], "--prompt-ids needs --weights"),
    (["--weights", "w", "--block-fixture", "--prompt-ids", "p"],
     "--prompt-ids cannot be combined with --block-fixture"),
    (["--fingerprint-dir", "d"], "--fingerprint-dir needs --weights or --block-fixture"),
    (["--block-fixture", "--block-fixture"], "--block-fixture was given more than once"),
    (["--weights", "a", "--weights", "b"], "--weights was given more than once"),
    (["--warmup", "1"], "--warmup, --repeats, and --cost-card need --arena-s1"),
    (["--arena-s1", "--block-fixture"], "--arena-s1 cannot be combined with --block-fixture"),
    (["--arena-s1"], "--arena-s1 needs --weights"),
    (["--arena-s1", "--weights", "w"], "--arena-s1 needs --prompt-ids"),
    (["--arena-s1", "--weights", "w", "--prompt-ids", "p"], "--arena-s1 needs --ref-ids"),
    (["--arena-s1", "--weights", "w", "--prompt-ids", "p", "--ref-ids", "r", "--warmup", "101"],
     "--warmup needs an integer from 0 to 100, got `101`"),
    (["--arena-s1", "--weights", "w", "--prompt-ids", "p", "--ref-ids", "r", "--repeats", "0"],
     "--repeats needs an integer from 1 to 100, got `0`"),
])
def test_usage_errors_exit_2(tmp_path, args, msg):
    code, out, err = run(args, tmp_path)
    assert code == 2
    assert out == ""
    assert err == f"MyOS: {msg}\n{USAGE}\n"
    assert not (tmp_path / "runs").exists()


def test_bad_ref_ids_exit_1(tmp_path):
    code, out, err = run(["--block-fixture", "--ref-ids", str(tmp_path / "absent.txt")], tmp_path)
    assert code == 1 and out == ""
    assert err.startswith("MyOS ref-ids: ")
    empty = tmp_path / "empty.txt"
    empty.write_text("  \n")
    code, _, err = run(["--ref-ids", str(empty)], tmp_path)
    assert code == 1 and "file is empty" in err
    bad = tmp_path / "bad.txt"
    bad.write_text("1 2 x")
    code, _, err = run(["--ref-ids", str(bad)], tmp_path)
    assert code == 1 and "`x` is not a u32" in err
