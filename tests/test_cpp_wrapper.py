"""The header-only C++ layer (include/uocr_moe.hpp) compiled into a program
against libuocr_moe.so: the reference's exception contract on the paths that
need no GPU (argument checks, checkpoint reading), and RAII ownership."""
import os
import shutil
import subprocess

import pytest

import uocr_moe as M

HERE = os.path.dirname(os.path.abspath(__file__))
INCLUDE = os.path.join(os.path.dirname(HERE), "include")

PROGRAM = r"""
#include <cstdio>
#include <stdexcept>
#include <string>
#include "uocr_moe.hpp"

template <typename E, typename F>
static void expect(const char* what, F&& f) {
  try {
    f();
    std::printf("%s: no exception\n", what);
  } catch (const E& e) {
    std::printf("%s: ok: %s\n", what, e.what());
  } catch (const std::exception& e) {
    std::printf("%s: wrong type: %s\n", what, e.what());
  }
}

int main(int argc, char** argv) {
  if (argc > 1 && std::string(argv[1]) == "format") {
    try {
      std::printf("format %d\n", static_cast<int>(uocr_b200::weight_format_from_env()));
    } catch (const std::invalid_argument& e) {
      std::printf("format error: %s\n", e.what());
    }
    return 0;
  }
  // ops.cu:655 throws invalid_argument above 128 experts; so does the wrapper
  expect<std::invalid_argument>("topk experts", [] {
    uocr_b200::expert_topk(nullptr, nullptr, 1, 129, 2, nullptr, nullptr);
  });
  expect<std::invalid_argument>("ffn k", [] {
    uocr_b200::expert_ffn_one(nullptr, nullptr, 64, 32, nullptr, nullptr, nullptr, nullptr, nullptr, 0, nullptr);
  });
  uocr_moe_desc bad{};
  expect<std::invalid_argument>("plan desc", [&] { uocr_b200::MoePlan p(bad); });
  expect<std::runtime_error>("missing file", [] { uocr_b200::Checkpoint c("/nonexistent/x.safetensors"); });
  {
    uocr_b200::Checkpoint ck(argv[1]);
    uocr_b200::Checkpoint moved(std::move(ck));
    std::printf("tensors %lld\n", static_cast<long long>(moved.size()));
    const uocr_tensor_view v = moved.at(argv[2]);
    std::printf("rank %d bytes %lld\n", v.rank, static_cast<long long>(v.bytes));
    expect<std::out_of_range>("absent tensor", [&] { moved.at("nope"); });
  }
  return 0;
}
"""


def test_cpp_wrapper_exceptions_and_ownership(tmp_path):
    cxx = shutil.which("g++") or shutil.which("c++")
    if cxx is None:
        pytest.skip("no C++ compiler")
    from test_checkpoint import write_moe_checkpoint
    idx, arrays = write_moe_checkpoint(tmp_path, [1], H=64, E=2, F=32, S=0)
    src = tmp_path / "wrap.cpp"
    src.write_text(PROGRAM)
    exe = tmp_path / "wrap"
    libdir = os.path.dirname(M.LIB_PATH)
    subprocess.run([cxx, "-std=c++17", "-Wall", "-Werror", "-I", INCLUDE, str(src), "-o", str(exe), "-L", libdir,
                    "-luocr_moe", f"-Wl,-rpath,{libdir}"], check=True)
    name = "model.layers.1.mlp.experts.1.gate_proj.weight"
    out = subprocess.run([str(exe), str(idx), name], check=True, capture_output=True, text=True).stdout.splitlines()
    assert out[0].startswith("topk experts: ok: uocr: ")
    assert out[1].startswith("ffn k: ok: uocr: expert_ffn_one: ")
    assert out[2].startswith("plan desc: ok: uocr: plan_create")
    assert out[3].startswith("missing file: ok: uocr: /nonexistent/x.safetensors: cannot open")
    assert out[4] == f"tensors {len(arrays)}"
    assert out[5] == f"rank 2 bytes {arrays[name].nbytes}"
    assert out[6] == "absent tensor: ok: uocr: no tensor named nope"

    for value, want in ((None, "format 0"), ("", "format 0"), ("bf16", "format 0"), ("int8", "format 1"),
                        ("fp32", "format error: GRPC_UOCR_WEIGHT_FORMAT must be one of bf16, int8")):
        env = {k: v for k, v in os.environ.items() if k != "GRPC_UOCR_WEIGHT_FORMAT"}
        if value is not None:
            env["GRPC_UOCR_WEIGHT_FORMAT"] = value
        r = subprocess.run([str(exe), "format"], check=True, capture_output=True, text=True, env=env)
        assert r.stdout.strip() == want, value
