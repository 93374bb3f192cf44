"""CPU checks of the C ABI boundary: the library builds, loads, and exports
every entry point include/shield_b200.h declares (no compute without a GPU)."""
from __future__ import annotations

import ctypes
import re
import subprocess
from pathlib import Path

import pytest

from llm_shield_b200 import _build, binding

REPO = Path(__file__).resolve().parent.parent


def declared_functions() -> list[str]:
    text = (REPO / "include" / "shield_b200.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(shield_[a-z_0-9]+)\s*\(", text)))


def test_header_declares_the_reference_boundary():
    names = declared_functions()
    for required in ("shield_open", "shield_close", "shield_set_config", "shield_upload_tensor",
                     "shield_score_batch", "shield_qmatmul", "shield_debug_block_dots", "shield_last_error"):
        assert required in names


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(str(_build.build_main()))
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing


def test_binding_covers_every_declared_symbol():
    assert sorted(binding.EXPORTS) == declared_functions()


def test_exports_are_c_linkage():
    out = subprocess.run(["nm", "-D", "--defined-only", str(_build.main_lib_path())], capture_output=True,
                         text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    for n in declared_functions():
        assert n in exported


def test_last_error_is_empty_before_any_failure():
    assert binding.lib().shield_last_error() in (b"", None)


def test_open_without_a_gpu_fails_loudly():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    h = ctypes.c_void_p()
    rc = binding.lib().shield_open(1, ctypes.byref(h))
    assert rc == binding.ERR_CUDA
    assert b"cuda" in binding.lib().shield_last_error().lower()


C_CLIENT = r"""
#include <stdio.h>
#include <string.h>
#include "shield_b200.h"

int main(void) {
    shield_ctx *ctx = NULL;
    shield_status rc = shield_open(1, &ctx);
    const char *msg = shield_last_error();
    if (rc == SHIELD_OK) { shield_close(ctx); return 0; }   /* a GPU is present */
    if (rc != SHIELD_ERR_CUDA || ctx != NULL || msg == NULL || strlen(msg) == 0) return 1;
    if (shield_set_prefix(NULL, NULL, 0) != SHIELD_ERR_ARG) return 2;
    if (shield_prefix_length(NULL, NULL) != SHIELD_ERR_ARG) return 3;
    printf("%d\n", rc);
    return 0;
}
"""


def test_header_is_plain_c_and_links_from_c(tmp_path):
    """What a cgo, P/Invoke or ctypes consumer sees: the header compiles as
    strict C99 and a C program links against the library and gets status
    codes back (no GPU here, so shield_open reports a CUDA failure)."""
    src = tmp_path / "client.c"
    src.write_text(C_CLIENT)
    lib = _build.build_main()
    exe = tmp_path / "client"
    subprocess.run(["gcc", "-std=c99", "-Wall", "-Wextra", "-Werror", "-pedantic", "-I", str(REPO / "include"),
                    str(src), "-o", str(exe), "-L", str(lib.parent), "-l:" + lib.name,
                    "-Wl,-rpath," + str(lib.parent)], check=True)
    import torch
    r = subprocess.run([str(exe)], capture_output=True, text=True)
    assert r.returncode == 0, (r.returncode, r.stdout, r.stderr)
    if not torch.cuda.is_available():
        assert r.stdout.strip() == str(binding.ERR_CUDA)
