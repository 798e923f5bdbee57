"""The C ABI from C: tests/c_abi/abi_consumer.c is compiled as plain C99
against include/semantica_b200.h and linked to libsemantica_b200.so, the way
a cgo binding would use them (every other test goes through ctypes).

Without a GPU: the header compiles as C with warnings as errors, the program
links and runs the device-free calls. On a GPU: the C program embeds a ragged
batch (its vectors equal the Python path's bit for bit: same library, same
kernels), runs the request pipeline, checks a reference error string and
builds, searches and round-trips a small int8 index."""
import os
import subprocess

import numpy as np
import pytest

import synth
from conftest import ROOT, TEST_VOCAB

SRC = os.path.join(ROOT, "tests", "c_abi", "abi_consumer.c")
BUILD = os.path.join(ROOT, "tests", "_build")
EXE = os.path.join(BUILD, "abi_consumer")


@pytest.fixture(scope="module")
def consumer():
    import _lib
    os.makedirs(BUILD, exist_ok=True)
    libdir = os.path.dirname(_lib.LIB_PATH)
    cmd = ["gcc", "-std=c99", "-Wall", "-Wextra", "-Werror", "-pedantic", "-O2",
           "-I", os.path.join(ROOT, "include"), SRC, "-o", EXE,
           "-L", libdir, "-lsemantica_b200", "-Wl,-rpath," + libdir]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    return EXE


def test_header_is_c99_and_library_links(consumer):
    r = subprocess.run([consumer, "link"], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr
    assert r.stdout.startswith("device_count rc=")


@pytest.mark.gpu
def test_c_consumer_embeds_like_python(consumer, model_path, gpu_model, tmp_path):
    lens = [64, 3, 200, 127, 512, 1]
    dims = [768, 512, 256, 128, 768, 64]
    ids, offs = synth.token_batch(31, lens, TEST_VOCAB)
    blob = np.concatenate([[len(lens)], offs, ids, dims]).astype(np.int32)
    ids_path, out_path = tmp_path / "ids.bin", tmp_path / "out.bin"
    blob.tofile(ids_path)
    r = subprocess.run([consumer, "run", model_path, str(ids_path), str(out_path)], capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0, (r.returncode, r.stdout, r.stderr)
    for line in ("ok embed", "ok pipeline", "ok error string", "ok index", "ok done"):
        assert line in r.stdout, r.stdout
    got = np.fromfile(out_path, dtype=np.float32)
    want = np.concatenate(gpu_model.forward_batch(ids, offs, dims))
    assert got.shape == want.shape
    np.testing.assert_array_equal(got, want)


def test_status_codes_match_header():
    # the Python binding's SEM_* status codes are the header's
    import re
    import _lib
    text = open(os.path.join(ROOT, "include", "semantica_b200.h")).read()
    codes = {m.group(1): int(m.group(2)) for m in re.finditer(r"#define (SEM_(?:OK|E[A-Z]+)) (\d+)", text)}
    assert codes["SEM_EINTERNAL"] == 6
    for name, value in codes.items():
        assert getattr(_lib, name) == value, name
