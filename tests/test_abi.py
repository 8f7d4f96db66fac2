# SPDX-License-Identifier: MIT
"""The C-ABI boundary, checked without a GPU.

* libdbs_cuda.so loads (no device needed) and exports every function include/*.h declares;
  it exports the reference's 17 dbs_cuda_* symbols (beamgrad 2.3.0 include/dbs_cuda.h:102-334);
* every struct has the reference layout: sizes and field offsets from the C compiler for this
  header, for the reference header when present, and for the ctypes mirror must agree;
* the headers compile as C (as tests/c_api_test.c does for the reference).
"""

from __future__ import annotations

import ctypes as C
import re
import subprocess
from pathlib import Path

import pytest

from beamgrad_b200 import _abi as A
from oracle import oracle

ROOT = Path(__file__).resolve().parents[1]
_REF = oracle.reference_dir()
REF_HEADER = _REF / "include" / "dbs_cuda.h" if _REF is not None else Path("reference-header-not-found")

STRUCTS = {
    "DBSCudaDecodeArgs": A.DecodeArgs,
    "DBSCudaDecodeOutputs": A.DecodeOutputs,
    "DBSCudaBeamState": A.BeamState,
    "DBSCudaBackwardInputs": A.BackwardInputs,
    "DBSCudaSearchOptions": A.SearchOptions,
}
# Structs of the engine's additions (include/dbs_cuda_b200.h).
B200_STRUCTS = {
    "DBSCudaVocabShardPlan": A.VocabShardPlan,
    "DBSCudaVocabShardBuffers": A.VocabShardBuffers,
    "DBSCudaVocabShardCall": A.VocabShardCall,
    "DBSCudaPoolOutputs": A.PoolOutputs,
    "DBSCudaPoolGradients": A.PoolGradients,
}


def declared_functions() -> list[str]:
    names = []
    for h in sorted((ROOT / "include").glob("*.h")):
        text = h.read_text()
        names += re.findall(r"DBS_CUDA_EXPORT\s+[\w\s\*]+?\b(dbs_cuda_\w+)\s*\(", text)
    return names


def test_library_loads_and_exports_every_declared_symbol():
    lib = A.load()
    declared = declared_functions()
    assert len(declared) >= 19
    for name in declared:
        assert hasattr(lib, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", str(A.LIB_PATH)], capture_output=True, text=True).stdout
    exported = set(re.findall(r" T (dbs_cuda_\w+)", out))
    assert set(declared) == exported


def test_reference_symbol_set_present():
    names = set(declared_functions())
    assert len(A.REFERENCE_SYMBOLS) == 17
    assert set(A.REFERENCE_SYMBOLS) <= names


def test_no_device_reports_unavailable_without_faulting():
    import torch

    if torch.cuda.is_available():
        pytest.skip("a device is present")
    assert A.load().dbs_cuda_available() == 0


def _c_layout(header: Path, tmp_path: Path, structs=STRUCTS) -> dict[str, list[int]]:
    fields = {name: [f[0] for f in cls._fields_] for name, cls in structs.items()}
    lines = ["#include <stdio.h>", "#include <stddef.h>", f'#include "{header}"', "int main(void) {"]
    for name, fs in fields.items():
        parts = [f"(int)sizeof({name})"] + [f"(int)offsetof({name}, {f})" for f in fs]
        fmt = " ".join(["%d"] * len(parts))
        lines.append(f'  printf("{name} {fmt}\\n", {", ".join(parts)});')
    lines += ["  return 0;", "}"]
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-std=c99", "-Wall", "-Werror", "-I", str(header.parent), "-o", str(exe), str(src)],
                   check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout
    return {line.split()[0]: [int(v) for v in line.split()[1:]] for line in out.strip().splitlines()}


def _ctypes_layout(structs=STRUCTS) -> dict[str, list[int]]:
    return {name: [C.sizeof(cls)] + [getattr(cls, f[0]).offset for f in cls._fields_] for name, cls in structs.items()}


def test_struct_layout_matches_ctypes(tmp_path):
    assert _c_layout(ROOT / "include" / "dbs_cuda.h", tmp_path) == _ctypes_layout()
    b200 = ROOT / "include" / "dbs_cuda_b200.h"
    assert _c_layout(b200, tmp_path, B200_STRUCTS) == _ctypes_layout(B200_STRUCTS)


@pytest.mark.skipif(not REF_HEADER.exists(), reason="reference tree not present")
def test_struct_layout_matches_reference_header(tmp_path):
    ours = _c_layout(ROOT / "include" / "dbs_cuda.h", tmp_path)
    ref = _c_layout(REF_HEADER, tmp_path)
    assert ours == ref


@pytest.mark.skipif(not REF_HEADER.exists(), reason="reference tree not present")
def test_constants_match_reference_header():
    pat = re.compile(r"#define\s+(DBS_CUDA_\w+)\s+(\d+)")
    ours = dict(pat.findall((ROOT / "include" / "dbs_cuda.h").read_text()))
    ref = dict(pat.findall(REF_HEADER.read_text()))
    ref.pop("DBS_CUDA_EXPORT", None)
    assert {k: ours.get(k) for k in ref} == ref


def test_headers_compile_as_c(tmp_path):
    src = tmp_path / "c_api.c"
    src.write_text('#include "dbs_cuda.h"\n#include "dbs_cuda_b200.h"\nint main(void) { DBSCudaDecodeArgs a = {0}; '
                   "return a.batch_size + DBS_CUDA_MAX_BEAM - 1024; }\n")
    subprocess.run(["gcc", "-std=c99", "-Wall", "-Werror", "-I", str(ROOT / "include"), "-c", str(src), "-o",
                    str(tmp_path / "c_api.o")], check=True)
