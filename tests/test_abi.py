"""The C-ABI boundary without a GPU: the library loads, exports every entry point that
include/tinferno_b200.h declares, the ctypes structs match the C layout, and argument errors
are reported as status codes (never exceptions or exits)."""
import ctypes as C
import os
import re
import subprocess
import tempfile

import pytest

from tinferno_b200 import native

HEADER = native.HEADER


def declared_functions():
    txt = open(HEADER).read()
    return re.findall(r"TF_API\s+[\w\s\*]+?\b(tf_\w+)\s*\(", txt)


def test_library_exports_every_declared_symbol():
    names = declared_functions()
    assert len(names) >= 20
    L = native.lib()
    for n in names:
        assert hasattr(L, n), n
    # and the ctypes signature table covers exactly the declared set
    assert sorted(n for n, _, _ in native.SIGNATURES) == sorted(names)


def test_struct_layout_matches_c(tmp_path):
    src = tmp_path / "layout.c"
    src.write_text(
        '#include <stdio.h>\n#include <stddef.h>\n#include "tinferno_b200.h"\n'
        "int main(void){printf(\"%zu %zu %zu %zu %zu %zu\\n\", sizeof(tf_tensor_desc),"
        " offsetof(tf_tensor_desc, data), offsetof(tf_tensor_desc, nbytes), sizeof(tf_hparams),"
        " sizeof(tf_options), offsetof(tf_hparams, eos));return 0;}\n")
    exe = tmp_path / "layout"
    subprocess.check_call(["gcc", "-I", os.path.dirname(HEADER), str(src), "-o", str(exe)])
    got = [int(v) for v in subprocess.check_output([str(exe)]).split()]
    want = [C.sizeof(native.TensorDesc), native.TensorDesc.data.offset, native.TensorDesc.nbytes.offset,
            C.sizeof(native.HParams), C.sizeof(native.Options), native.HParams.eos.offset]
    assert got == want


def test_errors_are_status_codes_without_gpu():
    L = native.lib()
    # null arguments are rejected before any device work
    h = C.c_void_p()
    assert L.tf_cuda_create(None, 0, None, None, C.byref(h)) != 0
    assert b"null" in L.tf_cuda_last_error(None)
    assert L.tf_cuda_decode(None, 0, 1, None, None) != 0
    assert L.tf_cuda_n_vocab(None) == -1
    assert L.tf_op_matmul(None, None, 99, None, 4, 32, 1, None) != 0  # unsupported type
    assert L.tf_op_matmul(None, None, 8, None, 4, 48, 1, None) != 0   # K not a block multiple


def test_describe_line():
    """Model::describe (src/model.cpp:91-105) as the host mirror formats it: the model's shape,
    then the GPU stage's settings."""
    from tinferno_b200 import synth
    from tinferno_b200.model import RunConfig, describe
    hp = native.HParams()
    c = synth.CFG0
    hp.n_vocab, hp.n_embd, hp.n_ff, hp.n_layer = c.n_vocab, c.n_embd, c.n_ff, c.n_layer
    hp.n_head, hp.n_kv_head = c.n_head, c.n_kv_head
    line = describe("llama", hp, synth.weight_bytes(c), RunConfig(max_seq=2048))
    assert line == ("arch=llama layers=16 dim=2048 heads=32/8 ff=8192 vocab=128256 weights=1313.25 MB "
                    "stage=b200 device=0 kv=f32 max_seq=2048 slots=1 graph=on decode=kernels")
