"""C-ABI library checks that need no GPU: it loads, exports every entry
point include/cascade_b200.h declares, its struct layouts match the ctypes
mirrors, and it fails cleanly (no crash) when no GPU is present."""
import ctypes as C
import os
import re
import subprocess

import pytest

from cascade_cpp import _lib as L

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
HEADER = os.path.join(ROOT, "include", "cascade_b200.h")


def header_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(cb_\w+)\s*\(", src)))


@pytest.fixture(scope="module")
def lib():
    if not os.path.exists(L.LIB_PATH):
        import sys
        sys.path.insert(0, os.path.join(ROOT, "kcj-cascade-v6_b200"))
        import build
        build.build()
    return L.load()


def test_header_declares_expected_surface():
    fns = header_functions()
    for f in ["cb_create", "cb_destroy", "cb_put_batch", "cb_get_batch", "cb_hash_batch",
              "cb_contains_batch", "cb_locate", "cb_evict", "cb_get_stats", "cb_clear",
              "cb_dht_attach", "cb_dht_barrier", "cb_dht_unique_id"]:
        assert f in fns


def test_library_exports_every_declared_symbol(lib):
    out = subprocess.run(["nm", "-D", "--defined-only", L.LIB_PATH], capture_output=True, text=True).stdout
    exported = set(re.findall(r"\bT (cb_\w+)", out))
    missing = [f for f in header_functions() if f not in exported]
    assert not missing, missing
    for f in header_functions():
        assert hasattr(lib, f)


def test_ctypes_signatures_cover_header():
    assert sorted(n for n, _, _ in L.SIGNATURES) == header_functions()


def test_constants_match_header():
    # every integer #define of the header has the same value in the ctypes layer
    headers = [HEADER] + [os.path.join(ROOT, "include", f) for f in os.listdir(os.path.join(ROOT, "include"))
                          if f.endswith(".h") and f != os.path.basename(HEADER)]
    defs = {}
    for h in headers:
        for name, val in re.findall(r"^#define\s+(CB_\w+)\s+(0x[0-9A-Fa-f]+|\d+)\b", open(h).read(), re.M):
            defs[name] = int(val, 0)
    assert len(defs) >= 24
    missing = [k for k in defs if not hasattr(L, k)]
    assert not missing, missing
    wrong = {k: (v, getattr(L, k)) for k, v in defs.items() if getattr(L, k) != v}
    assert not wrong, wrong


def test_struct_layouts_match_c(tmp_path):
    # every field of every ABI struct: the ctypes mirror's offset must be the
    # C compiler's offsetof, and the sizes must agree
    structs = [("cb_config", L.cb_config), ("cb_stats", L.cb_stats), ("cb_location", L.cb_location)]
    lines, want = [], []
    for cname, cls in structs:
        lines.append(f'printf("%zu\\n", sizeof({cname}));')
        want.append(C.sizeof(cls))
        for fname, _ in cls._fields_:
            lines.append(f'printf("%zu\\n", offsetof({cname}, {fname}));')
            want.append(getattr(cls, fname).offset)
    prog = tmp_path / "layout.c"
    prog.write_text('#include <stdio.h>\n#include <stddef.h>\n#include "cascade_b200.h"\n'
                    "int main(void){" + "".join(lines) + "return 0;}\n")
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-I", os.path.dirname(HEADER), str(prog), "-o", str(exe)], check=True)
    vals = [int(x) for x in subprocess.run([str(exe)], capture_output=True, text=True).stdout.split()]
    assert vals == want


def test_config_defaults(lib):
    cfg = L.cb_config()
    lib.cb_config_init(C.byref(cfg))
    assert cfg.gpu_capacity_bytes == 32 << 30  # DistributedConfig default
    assert cfg.dram_capacity_bytes == 64 << 30
    assert cfg.dedup_enabled == 1 and cfg.semantic_eviction == 1


def test_create_without_gpu_fails_cleanly(lib):
    import torch
    if torch.cuda.is_available():
        pytest.skip("GPU present")
    cfg = L.cb_config()
    lib.cb_config_init(C.byref(cfg))
    h = C.c_void_p()
    rc = lib.cb_create(C.byref(cfg), C.byref(h))
    assert rc != L.CB_OK and not h.value
    assert lib.cb_last_error(None)


def test_null_arguments_rejected(lib):
    assert lib.cb_put_batch(None, None, None, None, None, 1, 0, None, None, None) == L.CB_ERR_ARG
    assert lib.cb_get_batch(None, None, 1, None, None, 0, None, None, None) == L.CB_ERR_ARG
    assert lib.cb_destroy(None) == L.CB_OK


def test_product_never_imports_oracle():
    pkg = os.path.join(ROOT, "kcj-cascade-v6_b200")
    for dirpath, _, files in os.walk(pkg):
        for f in files:
            if f.endswith((".py", ".cu", ".cuh", ".cpp", ".hpp")):
                txt = open(os.path.join(dirpath, f)).read()
                assert "import oracle" not in txt and "from oracle" not in txt, f
                assert "sha256_oracle" not in txt, f


def test_integration_snippets_compile():
    # the C++ binding shown to maintainers compiles against this header
    pybind11 = pytest.importorskip("pybind11")
    import sysconfig
    src = os.path.join(ROOT, "tests", "snippets", "pybind_binding.cpp")
    r = subprocess.run(["g++", "-std=c++17", "-fsyntax-only", "-I", os.path.dirname(HEADER),
                        "-I", pybind11.get_include(), "-I", sysconfig.get_paths()["include"], src],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-2000:]


def test_plain_c_program_links_and_calls_the_library(lib, tmp_path):
    # the boundary from C: compile against the header, link the library,
    # call the entry points that need no GPU
    prog = tmp_path / "use.c"
    prog.write_text(r'''
#include <stdio.h>
#include <string.h>
#include "cascade_b200.h"
int main(void) {
  cb_config c;
  cb_config_init(&c);
  if (c.dedup_enabled != 1 || c.gpu_capacity_bytes != (32ull << 30)) return 1;
  uint8_t key[16];
  memset(key, 0, sizeof key);
  key[7] = 5;                                  /* first 8 bytes big-endian = 5 */
  if (cb_owner_rank(key, 4) != 1) return 2;    /* 5 mod 4 */
  if (cb_owner_rank(key, 0) != -1) return 3;   /* bad world */
  if (cb_put_batch(NULL, NULL, NULL, NULL, NULL, 1, CB_MEM_DEVICE, NULL, NULL, NULL) != CB_ERR_ARG) return 4;
  if (cb_destroy(NULL) != CB_OK) return 5;
  puts("ok");
  return 0;
}
''')
    exe = tmp_path / "use"
    libdir = os.path.dirname(L.LIB_PATH)
    subprocess.run(["gcc", "-std=c11", "-I", os.path.dirname(HEADER), str(prog), "-o", str(exe),
                    f"-L{libdir}", "-l:" + os.path.basename(L.LIB_PATH), f"-Wl,-rpath,{libdir}"], check=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True)
    assert r.returncode == 0 and r.stdout.strip() == "ok", (r.returncode, r.stdout, r.stderr)


def test_dht_route_and_owner_plan_without_a_gpu(lib):
    # the DHT's host-side routing and owner planning run without a GPU
    import numpy as np
    import cascade_cpp
    rng = np.random.default_rng(2)
    keys = rng.integers(0, 256, (50, 16), dtype=np.uint8)
    keys[10] = keys[3]  # a repeat inside the batch
    owner, order, counts = cascade_cpp.dht_route(keys, 3)
    want_owner = [int.from_bytes(k[:8].tobytes(), "big") % 3 for k in keys]
    assert owner.tolist() == want_owner
    assert counts.tolist() == [want_owner.count(r) for r in range(3)]
    assert order.tolist() == sorted(range(50), key=lambda i: (want_owner[i], i))
    p = cascade_cpp.DhtPlanner(1 << 20)
    status, loc = p.plan_put(keys, np.full(50, 4096, np.uint64), np.zeros(50, np.uint8))
    assert status.tolist() == [1 if i == 10 else 0 for i in range(50)]
    stored = loc[status == 0]
    assert len(set(stored.tolist())) == 49 and all(x % 256 == 0 for x in stored.tolist())
    # a second step: everything already held is a dedup hit; no room is a failure
    status2, _ = p.plan_put(keys[:5], np.full(5, 4096, np.uint64))
    assert status2.tolist() == [1] * 5
    big = rng.integers(0, 256, (1, 16), dtype=np.uint8)
    status3, _ = p.plan_put(big, np.array([2 << 20], np.uint64))
    assert status3.tolist() == [2]
    p.close()
