"""A plain C program against include/uocr_moe.h and libuocr_moe.so: the host
side of the checkpoint ABI (open, count, look up, error text) as a C caller
sees it. Host only; no GPU."""
import os
import shutil
import subprocess

import pytest

import safetensors_py as C
import uocr_moe as M

HERE = os.path.dirname(os.path.abspath(__file__))
INCLUDE = os.path.join(os.path.dirname(HERE), "include")

PROGRAM = r"""
#include <stdio.h>
#include <string.h>
#include "uocr_moe.h"

int main(int argc, char** argv) {
  uocr_checkpoint* ck = NULL;
  if (uocr_checkpoint_open(argv[1], &ck) != UOCR_OK) { printf("open failed: %s\n", uocr_last_error()); return 1; }
  int64_t n = 0;
  uocr_checkpoint_count(ck, &n);
  printf("tensors %lld\n", (long long)n);
  uocr_tensor_view v;
  if (uocr_checkpoint_tensor(ck, argv[2], &v) != UOCR_OK) { printf("lookup failed: %s\n", uocr_last_error()); return 2; }
  const unsigned short* bits = (const unsigned short*)v.data;
  printf("dtype %d rank %d shape %lld %lld bytes %lld first %u\n", v.dtype, v.rank, (long long)v.shape[0],
         (long long)v.shape[1], (long long)v.bytes, (unsigned)bits[0]);
  int rc = uocr_checkpoint_tensor(ck, "model.layers.9.mlp.gate.weight", &v);
  printf("absent rc %d: %s\n", rc, uocr_last_error());
  uocr_checkpoint_close(ck);
  printf("abi %d\n", uocr_abi_version());
  return 0;
}
"""


def test_c_program_reads_a_checkpoint(tmp_path):
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    from test_checkpoint import write_moe_checkpoint
    idx, arrays = write_moe_checkpoint(tmp_path, [1], H=64, E=4, F=32, S=64, shards=2)
    src = tmp_path / "host.c"
    src.write_text(PROGRAM)
    exe = tmp_path / "host"
    libdir = os.path.dirname(M.LIB_PATH)
    subprocess.run([cc, "-std=c99", "-I", INCLUDE, str(src), "-o", str(exe), "-L", libdir, "-luocr_moe",
                    f"-Wl,-rpath,{libdir}"], check=True)
    name = "model.layers.1.mlp.experts.2.down_proj.weight"
    out = subprocess.run([str(exe), str(idx), name], check=True, capture_output=True, text=True).stdout.splitlines()
    a = arrays[name]
    assert out[0] == f"tensors {len(arrays)}"
    assert out[1] == f"dtype {M.DTYPE_BF16} rank 2 shape {a.shape[0]} {a.shape[1]} bytes {a.nbytes} first {int(a.flat[0])}"
    assert out[2] == "absent rc 1: no tensor named model.layers.9.mlp.gate.weight"
    assert out[3] == "abi 5"
    bad = tmp_path / "bad.json"
    bad.write_text("{}")
    r = subprocess.run([str(exe), str(bad), name], capture_output=True, text=True)
    assert r.returncode == 1 and "no weight_map object" in r.stdout
