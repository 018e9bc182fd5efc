"""The C ABI as a C or C++ caller (a Rust FFI crate's view) sees it, on CPU:
include/kestrel_cuda.h compiles on its own as C11 and as C++17 with all
warnings as errors, a program that takes the address of every declared
entry point links against libkestrel_cuda.so (so each declaration has an
export of that name), and the calls that need no GPU behave as documented:
kc_init reports KC_ERR_CUDA without a device, kc_last_error(NULL) gives the
message, NULL contexts are KC_ERR_ARG, kc_gguf_inspect rejects a file that is
not GGUF, and kc_kernel_launches counts from zero."""
import os
import re
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "kestrel_cuda.h")
LIBDIR = os.path.join(ROOT, "kestrel_b200")


def header_symbols():
    txt = open(HEADER).read()
    return sorted(set(re.findall(r"^KC_API [^(]*?\b(kc_\w+)\(", txt, flags=re.M)))


PROGRAM = r"""
#include "kestrel_cuda.h"
#include <stdio.h>
#include <string.h>

typedef void (*entry_fn)(void);
static entry_fn const entry_points[] = {
%(ptrs)s
};

int main(int argc, char** argv) {
  (void)argc;
  int bad = 0;
  for (size_t i = 0; i < sizeof(entry_points) / sizeof(entry_points[0]); ++i)
    if (!entry_points[i]) bad = 1;
  if (kc_kernel_launches() != 0) bad = 2;
  kc_ctx* ctx = (kc_ctx*)0x1;
  int rc = kc_init(0, &ctx);
  const char* msg = kc_last_error(NULL);
  if (rc != KC_ERR_CUDA || ctx != NULL || !msg || !strstr(msg, "no CUDA device")) bad = 3;
  if (kc_sync(NULL) != KC_ERR_ARG) bad = 4;
  if (kc_moe_ffn_dev(NULL, 0, NULL, 0, NULL, NULL, NULL) != KC_ERR_ARG) bad = 5;
  char info[256];
  if (kc_gguf_inspect(argv[0], info, sizeof info) == KC_OK) bad = 6;  /* an ELF file, not GGUF */
  printf("%%d entry points, status %%d\n", (int)(sizeof(entry_points) / sizeof(entry_points[0])), bad);
  return bad;
}
"""


def build_and_run(tmp_path, compiler, std, ext):
    if not shutil.which(compiler):
        pytest.skip(f"{compiler} not found")
    from kestrel_b200 import cuda
    cuda.load_library()  # builds nothing; fails loudly if the library is missing
    src = tmp_path / f"caller.{ext}"
    ptrs = ",\n".join(f"    (entry_fn)&{s}" for s in header_symbols())
    src.write_text(PROGRAM % {"ptrs": ptrs})
    exe = tmp_path / f"caller_{compiler}"
    cmd = [compiler, f"-std={std}", "-Wall", "-Wextra", "-Werror", "-pedantic", "-I", os.path.dirname(HEADER),
           str(src), "-o", str(exe), "-L", LIBDIR, "-lkestrel_cuda", f"-Wl,-rpath,{LIBDIR}"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    r = subprocess.run([str(exe)], capture_output=True, text=True, env=env, timeout=120)
    assert r.returncode == 0, (r.returncode, r.stdout, r.stderr)
    assert f"{len(header_symbols())} entry points, status 0" in r.stdout


def test_header_compiles_and_links_as_c(tmp_path):
    build_and_run(tmp_path, "gcc", "c11", "c")


def test_header_compiles_and_links_as_cxx(tmp_path):
    build_and_run(tmp_path, "g++", "c++17", "cpp")
