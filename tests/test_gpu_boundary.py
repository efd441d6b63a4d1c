"""The drop-in boundary from the reference's side: oracle/_ref/b200_stage_test is a C++ program
compiled against the reference's own headers and objects (oracle/Makefile, target b200).  It
loads a GGUF with the reference's loader, builds the engine's tensor descriptors from
GGUF::tensors() and its hyper-parameters as Model::Model derives them (oracle/b200_stage.hpp,
the binding a maintainer adds to the reference), and runs the same prompt through the
reference's Model and through libtinferno_b200.so: greedy ids must be identical, logits within
1e-2 at every step, and the device greedy loop must reproduce the ids."""
import json
import os
import subprocess

import numpy as np
import pytest

from tinferno_b200 import synth

from conftest import GOLDEN, ROOT

pytestmark = pytest.mark.gpu

BIN = os.path.join(ROOT, "oracle", "_ref", "b200_stage_test")


def run(path, max_seq, n_decode, prompt):
    if not os.path.exists(BIN):
        pytest.skip("b200_stage_test not built (make -C oracle b200 where the reference sources are)")
    p = subprocess.run([BIN, path, str(max_seq), str(n_decode)] + [str(int(t)) for t in prompt],
                       capture_output=True, text=True, timeout=600)
    assert p.returncode in (0, 1), p.stderr
    res = json.loads(p.stdout.strip().splitlines()[-1])
    assert res["tokens_equal"] and res["generate_equal"] and res["n_pos_equal"], res
    assert res["max_abs_logit_diff"] < 1e-2, res
    assert p.returncode == 0
    return res


def test_reference_ci_model_through_the_binding():
    res = run(os.path.join(GOLDEN, "tiny_ci.gguf"), 64, 8, [1, 3, 5, 7])
    print(res)


@pytest.mark.parametrize("cfg", [synth.mini(synth.CFG1, 2, 4096), synth.mini(synth.CFG0, 2, 4096)],
                         ids=lambda c: c.name)
def test_synthetic_model_through_the_binding(cfg, model_cache):
    path = synth.model_path(cfg, model_cache)
    gold = np.load(os.path.join(GOLDEN, cfg.name + ".npz"))
    res = run(path, 256, len(gold["tokens"]), gold["prompt"])
    print(res)
