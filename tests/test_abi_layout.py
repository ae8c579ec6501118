"""The drop-in boundary without a GPU: ABI layout, exported symbols, the PJRT table itself."""
import ctypes
import json
import os
import re
import subprocess

import pytest

from conftest import LIB, ROOT

GOLDEN = os.path.join(ROOT, "tests", "golden")


def test_struct_offsets_match_upstream_pjrt_header():
    """Every struct of include/pjrt_b200_abi.h has the upstream v0.55 size and field offsets."""
    import sys
    sys.path.insert(0, GOLDEN)
    import abi_offsets
    fields = abi_offsets.struct_fields()
    ours = abi_offsets.measure('#include "include/pjrt_b200_abi.h"', fields, include_dirs=[ROOT])
    ref = json.load(open(os.path.join(GOLDEN, "pjrt_abi_offsets.json")))
    assert set(ref) == set(ours)
    bad = [(s, k, ours[s][k], ref[s][k]) for s in ref for k in ref[s] if ours[s].get(k) != ref[s][k]]
    assert not bad, bad[:10]
    assert ref["PJRT_Api"]["sizeof"] == 840


def _declared_symbols():
    names = set()
    for h in os.listdir(os.path.join(ROOT, "include")):
        text = open(os.path.join(ROOT, "include", h)).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        names |= set(re.findall(r"\b(GetPjrtApi|b200_\w+)\s*\(", text))
    return names


def test_library_exports_exactly_the_declared_entry_points(lib_path):
    out = subprocess.run(["nm", "-D", "--defined-only", lib_path], capture_output=True, text=True, check=True).stdout
    exported = {l.split()[-1] for l in out.splitlines() if " T " in l}
    declared = _declared_symbols()
    assert declared == exported, (declared ^ exported)
    lib = ctypes.CDLL(lib_path)
    for name in declared:
        assert getattr(lib, name) is not None


def test_api_table_version_and_slots(lib_path):
    from pjrt_b200 import pjrt
    api = pjrt.Api(lib_path)
    assert api.struct_size == 840
    assert api.version == (0, 55)
    # every slot is populated: real entry or an UNIMPLEMENTED stub
    assert all(api.fn[n] for n in pjrt.API_FIELDS)
    assert len(pjrt.API_FIELDS) == (840 - 40) // 8


def test_unimplemented_stub_reports_unimplemented(lib_path):
    from pjrt_b200 import pjrt
    api = pjrt.Api(lib_path)
    with pytest.raises(pjrt.PjrtError) as e:
        api.call("Executable_Serialize", pjrt.LoadedArgs(executable=None))
    assert e.value.code_name == "UNIMPLEMENTED"


def test_client_create_without_gpu_fails_cleanly(lib_path):
    """On a host with no CUDA device, Client_Create returns FAILED_PRECONDITION instead of crashing."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    from pjrt_b200 import pjrt
    with pytest.raises(pjrt.PjrtError) as e:
        pjrt.Client(pjrt.Api(lib_path))
    assert e.value.code_name == "FAILED_PRECONDITION"
