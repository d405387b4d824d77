"""The drop-in boundary as a foreign caller sees it: a plain C99 program
(what a Rust -sys crate, cgo or JNI would bind) compiled against
include/slmkv.h alone and linked to libslmkv.so, on the CPU (a host-only
context: bookkeeping and the scheduler, no device). It checks that the header
is valid C, that the C types and status codes are what the Python mirror
assumes, and the reference behaviours behind them: kv_cache.rs:27-41 (capacity
bounds), :302-321 (transactional truncation), the scheduler's prefill ->
first token -> decode -> finish sequence, and error messages through
slm_last_error."""

import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
LIB_DIR = ROOT / "small-lm-rs_b200" / "slmkv"

C_PROGRAM = r"""
#include <stdio.h>
#include <string.h>
#include "slmkv.h"

#define CHECK(cond) do { if (!(cond)) { printf("FAIL line %d: %s\n", __LINE__, #cond); return 1; } } while (0)

int main(void) {
  slm_config cfg;
  slm_ctx* ctx = NULL;
  int32_t seq = -1, len = -1, empty = -1, nd = 0, np = 0, nf = 0;
  int32_t dseq[4], pseq[4], pcnt[4], fst[4], gen[4], waiting = 0, running = 0;
  int64_t fid[4], preempt = 0, tokens = 0;
  slm_sched* s = NULL;
  slm_sched_config sc;

  memset(&cfg, 0, sizeof cfg);
  cfg.num_layers = 2; cfg.num_query_heads = 4; cfg.num_key_value_heads = 3;
  cfg.head_dimension = 64; cfg.context_length = 64; cfg.rope_theta = 10000.0f;
  cfg.num_blocks = 16; cfg.max_sequences = 2; cfg.kv_dtype = SLM_KV_F32;
  /* 4 query heads over 3 KV heads: rejected, message without a context */
  CHECK(slm_create(&cfg, -1, &ctx) == SLM_ERR_INVALID_CONFIGURATION);
  CHECK(ctx == NULL && strlen(slm_last_error(NULL)) > 0);

  cfg.num_key_value_heads = 2;
  CHECK(slm_create(&cfg, -1, &ctx) == SLM_OK && ctx != NULL);
  CHECK(slm_seq_create(ctx, 65, &seq) != SLM_OK);          /* beyond context_length */
  CHECK(slm_seq_create(ctx, 32, &seq) == SLM_OK && seq >= 0);
  CHECK(slm_seq_length(ctx, seq, &len) == SLM_OK && len == 0);
  CHECK(slm_seq_is_empty(ctx, seq, &empty) == SLM_OK && empty == 1);
  CHECK(slm_seq_truncate_all(ctx, seq, 5) == SLM_ERR_INVALID_INPUT);  /* longer than cached */
  CHECK(strlen(slm_last_error(ctx)) > 0);
  CHECK(slm_seq_free(ctx, seq) == SLM_OK);
  CHECK(slm_seq_free(ctx, seq) != SLM_OK);                  /* unknown id now */

  sc.max_running = 2; sc.max_prefill_tokens = 8;
  CHECK(slm_sched_create(ctx, &sc, &s) == SLM_OK);
  CHECK(slm_sched_submit(s, 7, 10, 2) == SLM_OK);
  CHECK(slm_sched_submit(s, 7, 10, 2) == SLM_ERR_INVALID_INPUT);  /* duplicate id */
  CHECK(slm_sched_submit(s, 8, 60, 10) == SLM_ERR_CAPACITY);       /* 70 > context */
  /* step 1: 8 of the 10 prompt tokens */
  CHECK(slm_sched_plan(s, &nd, dseq, &np, pseq, pcnt) == SLM_OK && nd == 0 && np == 1 && pcnt[0] == 8);
  fst[0] = SLM_OK;
  CHECK(slm_sched_commit(s, NULL, fst, &nf, fid, fst + 1, gen) == SLM_OK && nf == 0);
  /* step 2: the prompt's last 2 tokens, which yield the first output token */
  CHECK(slm_sched_plan(s, &nd, dseq, &np, pseq, pcnt) == SLM_OK && nd == 0 && np == 1 && pcnt[0] == 2);
  CHECK(slm_sched_commit(s, NULL, fst, &nf, fid, fst + 1, gen) == SLM_OK && nf == 0);
  /* step 3: one decode token, the second and last output token */
  CHECK(slm_sched_plan(s, &nd, dseq, &np, pseq, pcnt) == SLM_OK && nd == 1 && np == 0);
  CHECK(slm_sched_commit(s, fst, NULL, &nf, fid, fst + 1, gen) == SLM_OK);
  CHECK(nf == 1 && fid[0] == 7 && fst[1] == SLM_OK && gen[0] == 2);
  CHECK(slm_sched_counts(s, &waiting, &running, &preempt, &tokens) == SLM_OK);
  CHECK(waiting == 0 && running == 0 && preempt == 0 && tokens == 2);
  CHECK(slm_sched_plan(s, &nd, dseq, &np, pseq, pcnt) == SLM_OK && nd == 0 && np == 0);
  CHECK(slm_sched_destroy(s) == SLM_OK);
  CHECK(slm_destroy(ctx) == SLM_OK);
  printf("ok\n");
  return 0;
}
"""


@pytest.fixture(scope="module")
def c_program(tmp_path_factory):
    import slmkv

    slmkv.lib()  # builds libslmkv.so if it is missing
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    d = tmp_path_factory.mktemp("c_abi")
    src, exe = d / "abi.c", d / "abi"
    src.write_text(C_PROGRAM)
    subprocess.run([cc, "-std=c99", "-Wall", "-Wextra", "-Werror", "-pedantic", f"-I{ROOT / 'include'}",
                    str(src), "-o", str(exe), f"-L{LIB_DIR}", "-lslmkv", f"-Wl,-rpath,{LIB_DIR}"],
                   check=True, capture_output=True, text=True)
    return exe


def test_header_compiles_as_c99_and_the_abi_works_from_c(c_program):
    r = subprocess.run([str(c_program)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0 and r.stdout.strip().endswith("ok"), r.stdout + r.stderr
