"""The C ABI from a plain C program (tests/c/select_main.c, INTEGRATION.md's C
example): it compiles and links against libttn.so on the CPU; on a B200 it runs the
class-aware selection through ttn_malloc / ttn_memcpy_async / ttn_select_f16 /
ttn_free with no PyTorch in its process, bit-exact against the selection oracle."""
from __future__ import annotations

import shutil
import subprocess
from pathlib import Path

import numpy as np
import pytest
import torch

import bench_configs as bc
from oracle import select as osel

ROOT = Path(__file__).resolve().parent.parent
LIB_DIR = ROOT / "thintnpu_b200"


def _build(tmp_path: Path) -> Path:
    gcc = shutil.which("gcc")
    if gcc is None:
        pytest.skip("gcc is not on PATH")
    exe = tmp_path / "select_main"
    cmd = [gcc, "-std=c11", "-Wall", "-Wextra", "-Werror", f"-I{ROOT / 'include'}",
           str(ROOT / "tests" / "c" / "select_main.c"), f"-L{LIB_DIR}", "-lttn", f"-Wl,-rpath,{LIB_DIR}",
           "-o", str(exe)]
    done = subprocess.run(cmd, capture_output=True, text=True)
    assert done.returncode == 0, done.stderr
    return exe


def test_c_caller_compiles_and_links(tmp_path):
    assert _build(tmp_path).exists()


@pytest.mark.gpu
@pytest.mark.parametrize("b,k", [(3, 300), (1, 8400)])
def test_c_caller_selects_bit_exact(tmp_path, b, k):
    exe = _build(tmp_path)
    logits = bc.config5_logits(b, 70 + b, "cpu")                 # [b, 84, 8400] fp16
    decoded = logits.transpose(1, 2).contiguous()                 # [b, 8400, 84]
    (tmp_path / "in.bin").write_bytes(decoded.view(torch.int16).numpy().tobytes())
    done = subprocess.run([str(exe), str(tmp_path / "in.bin"), str(tmp_path / "out.bin"), str(b), "8400", "80",
                           str(k)], capture_output=True, text=True)
    assert done.returncode == 0, done.stderr
    rows = min(k, 8400)
    got = np.frombuffer((tmp_path / "out.bin").read_bytes(), dtype=np.uint32).reshape(b, rows, 6)
    scores = decoded.clone()
    scores[..., 4:] = torch.sigmoid(scores[..., 4:])
    bits = scores.view(torch.int16).numpy().view(np.uint16)
    want = osel.select(bits, k)["output"]
    assert np.array_equal(got, want)
