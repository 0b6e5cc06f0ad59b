"""The ggml adapter's ggml-free half on the CPU.

xdna.cpp_b200/ggml/ggml-b200-adapter.cpp (built only against a ggml tree)
hands ggml graphs to the compat ABI through include/ggml-b200-convert.h.
tests/cpp/ggml_convert_check.cpp compiles that header with a stand-in
tensor type, converts a small graph (MUL_MAT nodes among others, a 4-D node,
a host op id that collides with the compat MUL_MAT id) and passes the records
to the library's claim predicate; no GPU is needed.
"""
import os
import subprocess

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_convert_header_with_stand_in_tensors(G, tmp_path):
    exe = tmp_path / "ggml_convert_check"
    lib_dir = os.path.join(ROOT, "xdna.cpp_b200")
    subprocess.run(["g++", "-std=c++17", "-O1", "-Wall", "-Wextra", "-Werror", "-I", os.path.join(ROOT, "include"),
                    os.path.join(ROOT, "tests", "cpp", "ggml_convert_check.cpp"), "-L", lib_dir, "-lggml-b200",
                    "-Wl,-rpath," + lib_dir, "-o", str(exe)], check=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0, r.stderr
    assert "ok" in r.stdout


def test_adapter_source_is_gated_on_a_ggml_tree():
    """The adapter compiles only with ggml's headers (XDNA_LLAMA_CPP_DIR), as
    the reference builds its plugin only when it finds them."""
    src = open(os.path.join(ROOT, "xdna.cpp_b200", "ggml", "ggml-b200-adapter.cpp")).read()
    for sym in ("ggml_backend_init", "ggml_backend_score", "ggml_backend_b200_graph_compute", "ggml_graph_node",
                "ggml_backend_buffer_init", "ggml_backend_xdna_compute_graph"):
        assert sym in src, sym
    build = open(os.path.join(ROOT, "xdna.cpp_b200", "build.py")).read()
    assert "XDNA_LLAMA_CPP_DIR" in build
