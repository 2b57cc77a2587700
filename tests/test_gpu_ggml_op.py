"""The ggml-shaped fused decode (sp_ggml_attn_decode) called from a C program
compiled against the public headers (tests/c/ggml_decode_check.c), the way a
ggml-cuda backend op replacing the reference's fused-KQ op
(patches/llama-cpp-b8861-full-engine.patch:393-410) would call it: padded
F32 query and output views, GQA 4.  The output is checked against the CPU
oracle's attention over the same packed slots (queries rounded to fp16, as
the op stages them), within 1e-3 relative L2."""
import os
import subprocess
from pathlib import Path

import numpy as np
import pytest

import oracle as O

ROOT = Path(__file__).resolve().parent.parent
PKG = ROOT / "shannon-prime-llama_b200"
CUDA = os.environ.get("CUDA_HOME", "/usr/local/cuda")


def _build(tmp_path, built_lib):
    exe = tmp_path / "ggml_decode_check"
    cmd = ["gcc", "-std=c11", "-O1", "-Wall", "-Werror", f"-I{ROOT / 'include'}", f"-I{CUDA}/include",
           str(ROOT / "tests" / "c" / "ggml_decode_check.c"), "-o", str(exe),
           f"-L{built_lib.parent}", "-lshannon_prime_b200", f"-L{CUDA}/lib64", "-lcudart",
           f"-Wl,-rpath,{built_lib.parent}", f"-Wl,-rpath,{CUDA}/lib64"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    return exe


def test_c_client_compiles_against_headers(built_lib, tmp_path):
    _build(tmp_path, built_lib)


@pytest.mark.gpu
def test_ggml_op_from_c_against_oracle(cuda, built_lib, tmp_path):
    exe = _build(tmp_path, built_lib)
    out = tmp_path / "dump.bin"
    r = subprocess.run([str(exe), str(out)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0 and "GGML_DECODE_OK" in r.stdout, r.stdout + r.stderr
    raw = out.read_bytes()
    L, H, G, HD, T, MS, KB, VB = np.frombuffer(raw[:32], np.int32)
    scale = float(np.frombuffer(raw[32:36], np.float32)[0])
    off = 36
    nq = H * G
    q = np.frombuffer(raw[off:off + nq * HD * 4], np.float32).reshape(nq, HD)
    off += nq * HD * 4
    got = np.frombuffer(raw[off:off + nq * HD * 4], np.float32).reshape(nq, HD)
    off += nq * HD * 4
    ks = np.frombuffer(raw[off:off + H * MS * KB], np.uint8).reshape(H, MS, KB)
    off += H * MS * KB
    vs = np.frombuffer(raw[off:off + H * MS * VB], np.uint8).reshape(H, MS, VB)
    ref = O.attn_decode(ks, vs, HD, [5, 5, 4, 3], [3], True, q.astype(np.float16), T, scale)
    err = np.linalg.norm(got - ref) / np.linalg.norm(ref)
    assert err <= 1e-3, err
