"""The C ABI from a C99 program: include/kvquant_b200.h compiles as plain C, the
library links, and the calls that need no GPU (version, workspace queries, argument
checks) behave as declared. No GPU needed."""
import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
LIB = ROOT / "kvquant-paper-repro_b200" / "kvquant" / "_lib" / "libkvquant_b200.so"

PROGRAM = r"""
#include <stdio.h>
#include <string.h>
#include "kvquant_b200.h"

int main(void) {
  int fails = 0;
  if (kvq_version() < 100) { puts("version"); ++fails; }
  if (kvq_decode_attention_workspace(1, 32, 1, 4096) < (size_t)2 * 32 * 4096 * 4) {
    puts("decode workspace"); ++fails;
  }
  if (kvq_fit_codebook_workspace(1 << 20) <= kvq_fit_codebook_workspace(1)) {
    puts("codebook workspace"); ++fails;
  }
  /* invalid arguments are rejected before any launch, with a message */
  if (kvq_fit_codebook(NULL, NULL, 10, 3, 2, NULL, NULL, 0, NULL, NULL) != KVQ_ERR_INVALID ||
      strlen(kvq_last_error()) == 0) {
    puts("codebook check"); ++fails;
  }
  if (kvq_rope_apply(NULL, NULL, NULL, NULL, 1, 1, 1, 3, 0, 1, NULL) != KVQ_ERR_INVALID) {
    puts("rope check"); ++fails;
  }
  if (kvq_merge_shards(NULL, NULL, 0, 4, NULL, NULL) != KVQ_ERR_INVALID) {
    puts("merge check"); ++fails;
  }
  printf("fails=%d\n", fails);
  return fails;
}
"""


@pytest.mark.skipif(shutil.which("gcc") is None, reason="no C compiler")
def test_c_program_builds_links_and_runs(tmp_path):
    if not LIB.exists():
        pytest.skip("library not built")
    src = tmp_path / "consumer.c"
    src.write_text(PROGRAM)
    exe = tmp_path / "consumer"
    subprocess.run(["gcc", "-std=c99", "-Wall", "-Werror", "-pedantic", "-I", str(ROOT / "include"),
                    str(src), "-o", str(exe), "-L", str(LIB.parent), "-lkvquant_b200",
                    f"-Wl,-rpath,{LIB.parent}"], check=True, capture_output=True, text=True)
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert run.returncode == 0, run.stdout + run.stderr
    assert "fails=0" in run.stdout
