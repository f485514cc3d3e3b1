"""The device variant of ennf2c (``spinn_b200/ennf2c_cuda.py``): generated sources build on
the CPU; on a B200 the generated program's output matches the reference runtime (O-fix) on
the same image and input (``input[i] = i / 1000``, as ennf2c's main_test.c feeds it)."""
import os
import re
import subprocess

import numpy as np
import pytest

from conftest import rel_l2

DRIVER_C = r"""
/* test driver: input file -> model_run -> output file, through the generated model.c */
#include <stdio.h>
#include <stdlib.h>
#include "model.h"
int main(int argc, char **argv) {
    float *in = (float *)malloc(MODEL_INPUT_SIZE), *out = (float *)malloc(MODEL_OUTPUT_SIZE);
    FILE *f = fopen(argv[1], "rb");
    if (!f || fread(in, 1, MODEL_INPUT_SIZE, f) != MODEL_INPUT_SIZE) return 2;
    fclose(f);
    model_init();
    int rc = model_run(in, out);
    if (rc == 0) rc = model_run(in, out);  /* a second run replays the same plan */
    if (rc != 0) { fprintf(stderr, "model_run %d\n", rc); return 3; }
    f = fopen(argv[2], "wb");
    fwrite(out, 1, MODEL_OUTPUT_SIZE, f);
    fclose(f);
    model_free();
    return 0;
}
"""


def _model():
    from spinn_b200 import ennf, netdef
    g = netdef.resnet(50, batch=1, image=64, width=16, seed=5)
    return ennf.convert(g)


def _build(tmp_path, image):
    from spinn_b200 import ennf2c_cuda
    out = tmp_path / "gen"
    ennf2c_cuda.generate(image, str(out))
    r = subprocess.run(["make", "-C", str(out)], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    (out / "driver.c").write_text(DRIVER_C)
    here = os.path.dirname(os.path.abspath(__file__))
    root = os.path.dirname(here)
    lib = os.path.join(root, "spinn_b200")
    r = subprocess.run(["gcc", "-O2", "-Wall", "-I", str(out), "-I", os.path.join(root, "include"), "-o",
                        str(out / "driver"), str(out / "driver.c"), str(out / "model.c"), str(out / "model_blob.S"),
                        "-L" + lib, "-lspinn_cuda", "-Wl,-rpath," + lib], capture_output=True, text=True, cwd=out)
    assert r.returncode == 0, r.stderr
    return out


def test_generated_sources_build(tmp_path):
    from spinn_b200 import ennf
    image = _model()
    m = ennf.read(image)
    out = _build(tmp_path, image)
    h = (out / "model.h").read_text()
    macros = dict(re.findall(r"#define (MODEL_\w+)\s+(\d+)", h))
    t_in, t_out = m.tensors[m.inputs[0]], m.tensors[m.outputs[0]]
    assert int(macros["MODEL_INPUT_ELEMS"]) == t_in.elem_count == 3 * 64 * 64
    assert int(macros["MODEL_OUTPUT_ELEMS"]) == t_out.elem_count == 1000
    assert int(macros["MODEL_INPUT_SIZE"]) == 4 * t_in.elem_count
    assert int(macros["MODEL_NUM_NODES"]) == len(m.nodes)
    assert (out / "model.ennf").read_bytes() == image
    assert (out / "main_test").exists() and (out / "driver").exists()


def test_malformed_image_is_rejected(tmp_path):
    from spinn_b200 import ennf2c_cuda
    with pytest.raises(ValueError):
        ennf2c_cuda.generate(b"\0" * 256, str(tmp_path / "bad"))


@pytest.mark.gpu
def test_generated_program_matches_reference(tmp_path, cuda_lib, ref_oracle):
    image = _model()
    out = _build(tmp_path, image)
    x = (np.arange(3 * 64 * 64, dtype=np.float32) / 1000.0).astype(np.float32)
    (tmp_path / "in.bin").write_bytes(x.tobytes())
    r = subprocess.run([str(out / "driver"), str(tmp_path / "in.bin"), str(tmp_path / "out.bin")],
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    y = np.frombuffer((tmp_path / "out.bin").read_bytes(), np.float32)
    p = tmp_path / "model.ennf"
    p.write_bytes(image)
    from spinn_b200 import ennf
    m = ennf.read(image)
    ref = ref_oracle.run_model(str(p), x.reshape(1, 3, 64, 64))[m.outputs[0]].reshape(-1)
    assert np.isfinite(y).all()
    assert rel_l2(y, ref) <= 2e-3, rel_l2(y, ref)
    assert int(np.argmax(y)) == int(np.argmax(ref))
    # the generated main_test.c: same input, prints the first ten outputs
    r = subprocess.run([str(out / "main_test")], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    vals = np.array([float(v) for v in r.stdout.split("Generated Result:")[1].split()], np.float32)
    assert vals.shape == (10,)
    assert np.allclose(vals, y[:10], atol=1e-5 + 1e-6 * np.abs(y[:10]).max())
