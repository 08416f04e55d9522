"""The per-context address cache behind qg_layer_slice_forward_static
(csrc/qg_ctx_cache.h), exercised on the CPU: a small C++ driver compiled with g++
feeds it context ids and counts the lookups."""

import subprocess

import pytest

from conftest import REPO

DRIVER = r"""
#include <cstdio>
#include "qg_ctx_cache.h"
static int lookups = 0;
static char slots[8];
int main() {
  qg::CtxAddressCache<4> cache;
  void* p = nullptr;
  auto look = [](void** out) { *out = &slots[lookups++ % 8]; return 0; };
  auto fail = [](void** out) { *out = nullptr; return 700; };
  int rc = cache.get(0, 11, look, &p);            // first call in context 11: lookup
  if (rc != 0 || lookups != 1 || p != &slots[0]) return 1;
  rc = cache.get(0, 11, look, &p);                // same context: cached
  if (rc != 0 || lookups != 1 || p != &slots[0]) return 2;
  rc = cache.get(0, 12, look, &p);                // context re-created (reset): lookup again
  if (rc != 0 || lookups != 2 || p != &slots[1]) return 3;
  rc = cache.get(1, 12, look, &p);                // other device: its own entry
  if (rc != 0 || lookups != 3 || p != &slots[2]) return 4;
  rc = cache.get(0, 12, look, &p);                // device 0 still cached for context 12
  if (rc != 0 || lookups != 3 || p != &slots[1]) return 5;
  rc = cache.get(0, 13, fail, &p);                // a failing lookup propagates, keeps entry
  if (rc != 700) return 6;
  rc = cache.get(0, 12, look, &p);
  if (rc != 0 || lookups != 3 || p != &slots[1]) return 7;
  if (cache.get(4, 12, look, &p) != -1 || cache.get(-1, 12, look, &p) != -1) return 8;
  std::puts("ok");
  return 0;
}
"""


def test_context_cache_relooks_up_per_context(tmp_path):
    src = tmp_path / "drv.cpp"
    src.write_text(DRIVER)
    exe = tmp_path / "drv"
    inc = REPO / "local-ai-gpu-acceleration_b200" / "csrc"
    try:
        subprocess.run(["g++", "-std=c++17", "-O1", f"-I{inc}", str(src), "-o", str(exe)],
                       check=True, capture_output=True, text=True)
    except FileNotFoundError:
        pytest.skip("no host C++ compiler")
    res = subprocess.run([str(exe)], capture_output=True, text=True)
    assert res.returncode == 0 and res.stdout.strip() == "ok", res.returncode
