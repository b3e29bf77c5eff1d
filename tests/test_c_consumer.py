"""The C ABI from C: tests/c/abi_consumer.c is compiled with gcc against
include/har_cuda.h alone and linked to libhar_cuda.so, then run (CPU only:
context creation must fail closed without a GPU; a GGUF directory is read
through the ABI)."""
import os
import shutil
import subprocess

import numpy as np
import pytest

import har_cuda
from gguf_writer import write_gguf

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_c_consumer_links_and_fails_closed(tmp_path):
    gcc = shutil.which("gcc")
    if gcc is None:
        pytest.skip("no C compiler")
    har_cuda.load_library()  # the library exists (built in-tree)
    libdir = os.path.dirname(har_cuda.LIB_PATH)
    exe = tmp_path / "abi_consumer"
    subprocess.run([gcc, "-std=c11", "-Wall", "-Werror", "-I", os.path.join(ROOT, "include"),
                    os.path.join(ROOT, "tests", "c", "abi_consumer.c"), "-o", str(exe),
                    "-L", libdir, "-lhar_cuda", "-Wl,-rpath," + libdir], check=True)
    p = tmp_path / "one.gguf"
    write_gguf(p, [], [("blk.0.ffn_down_exps.weight", [512, 4, 2], 12,
                        np.zeros(2 * 4 * 2 * 144, np.uint8))])
    r = subprocess.run([str(exe), str(p)], capture_output=True, text=True, timeout=120)
    out = r.stdout.strip()
    assert r.returncode == 0, out + r.stderr
    fields = dict(kv.split("=", 1) for kv in out.split())
    assert fields["abi"] == "1"
    import torch
    if not torch.cuda.is_available():
        assert int(fields["ctx_status"]) != har_cuda.OK
    assert fields["version"] == "3" and fields["tensors"] == "1" and fields["type"] == "12"
    assert fields["name"] == "blk.0.ffn_down_exps.weight" and fields["rank"] == "3"
    assert fields["payload"] == str(2 * 4 * 2 * 144)
