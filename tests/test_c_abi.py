"""The C ABI from C: include/mold_b200.h compiles as strict C11 (what a Rust / cgo binding
generator sees), and a C program linked against libmold_b200.so gets the documented status
codes and messages without a GPU."""
import os
import shutil
import subprocess

import pytest

from mold_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

C_SRC = r"""
#include <stdio.h>
#include <string.h>
#include "mold_b200.h"

static int fails = 0;
#define EXPECT(cond, what) do { if (!(cond)) { printf("FAIL %s: %s\n", what, mb_last_error()); fails++; } } while (0)

int main(void) {
  EXPECT(mb_version() > 0, "version");
  mb_weight* w = NULL;
  unsigned char raw[144] = {0};
  EXPECT(mb_weight_create(10, 1, 256, raw, sizeof raw, 0, &w) == MB_ERR_UNSUPPORTED, "Q2_K unsupported");
  EXPECT(strstr(mb_last_error(), "unsupported ggml type") != NULL, "message");
  EXPECT(mb_weight_create(MB_GGML_Q4_K, 1, 100, raw, sizeof raw, 0, &w) == MB_ERR_INVALID, "K % 256");
  EXPECT(mb_dequant(NULL, NULL, MB_DT_F32, NULL) == MB_ERR_INVALID, "NULL weight");
  EXPECT(mb_weight_lora_merge(NULL, 0, 1, NULL, NULL, 1, 1.0f, NULL) == MB_ERR_INVALID, "NULL lora weight");
  char buf[64];
  int64_t n = 0;
  EXPECT(mb_gguf_inspect("/nonexistent/file.gguf", buf, sizeof buf, &n) == MB_ERR_INVALID, "missing gguf");
  mb_flux_config cfg;
  memset(&cfg, 0, sizeof cfg);
  cfg.in_channels = 64; cfg.vec_in_dim = 768; cfg.context_in_dim = 4096; cfg.hidden_size = 3000;
  cfg.mlp_hidden = 12000; cfg.num_heads = 24; cfg.depth = 1; cfg.depth_single = 1;
  cfg.axes_dim[0] = 16; cfg.axes_dim[1] = 56; cfg.axes_dim[2] = 56; cfg.theta = 10000; cfg.guidance_embed = 1;
  mb_flux* m = NULL;
  EXPECT(mb_flux_create(&cfg, 512, 4096, &m) == MB_ERR_UNSUPPORTED, "head_dim 125");
  printf("%s\n", fails ? "FAILED" : "OK");
  return fails;
}
"""


@pytest.fixture(scope="module")
def cc():
    gcc = shutil.which("gcc") or shutil.which("cc")
    if gcc is None:
        pytest.skip("no C compiler")
    return gcc


def test_header_is_strict_c11(cc, tmp_path):
    src = tmp_path / "h.c"
    src.write_text('#include "mold_b200.h"\nint main(void) { return mb_version() > 0 ? 0 : 1; }\n')
    r = subprocess.run([cc, "-std=c11", "-Wall", "-Wextra", "-pedantic", "-Werror", "-fsyntax-only",
                        "-I", os.path.join(ROOT, "include"), str(src)], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr


def test_c_program_gets_status_codes(cc, tmp_path):
    src = tmp_path / "t.c"
    src.write_text(C_SRC)
    exe = tmp_path / "t"
    libdir = os.path.dirname(_lib.LIB_PATH)
    r = subprocess.run([cc, "-std=c11", "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe), "-L", libdir,
                        "-lmold_b200", "-Wl,-rpath," + libdir], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert run.returncode == 0 and "OK" in run.stdout, run.stdout + run.stderr
