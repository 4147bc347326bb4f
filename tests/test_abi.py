"""The C ABI boundary without a GPU: libplm_native.so loads, exports every entry point include/plm_native.h declares,
the ctypes mirrors of its structs have the C layout (sizes and field offsets compiled by gcc), and calls fail with a
status (never a crash or a silent fallback) when no sm_100a device is present."""

from __future__ import annotations

import ctypes
import re
import subprocess
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "plm_native.h"


def _declared_functions() -> list[str]:
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^int (plm_\w+)\(", text, flags=re.M)))


def test_library_exports_every_declared_symbol():
    from plm import native

    lib = native.library()
    declared = _declared_functions()
    assert len(declared) >= 20
    for name in declared:
        assert hasattr(lib, name), f"{name} is declared but not exported"
    assert sorted(native.exported_symbols()) == declared, "ctypes signatures must cover exactly the header"
    assert lib.plm_abi_version() == 8


STRUCTS = ["plm_gemm_epilogue", "plm_gemm_desc", "plm_bookkeeping", "plm_verify_desc", "plm_attention_desc",
           "plm_kv_append_desc", "plm_add_rmsnorm_desc", "plm_model_desc", "plm_weight_ptrs", "plm_round_desc",
           "plm_state_ptrs", "plm_icdf_desc", "plm_commit_desc", "plm_ptp_desc"]
MIRRORS = {"plm_gemm_epilogue": "GemmEpilogue", "plm_gemm_desc": "GemmDesc", "plm_bookkeeping": "Bookkeeping",
           "plm_verify_desc": "VerifyDesc", "plm_attention_desc": "AttentionDesc",
           "plm_kv_append_desc": "KvAppendDesc", "plm_add_rmsnorm_desc": "AddRmsNormDesc",
           "plm_model_desc": "ModelDesc", "plm_weight_ptrs": "WeightPtrs", "plm_round_desc": "RoundDesc",
           "plm_state_ptrs": "StatePtrs", "plm_icdf_desc": "IcdfDesc", "plm_commit_desc": "CommitDesc",
           "plm_ptp_desc": "PtpDesc"}


def test_ctypes_structs_match_c_layout(tmp_path):
    from plm import native

    lines = ['#include <stdio.h>', '#include <stddef.h>', f'#include "{HEADER}"', "int main(void) {"]
    for struct in STRUCTS:
        mirror = getattr(native, MIRRORS[struct])
        lines.append(f'  printf("{struct} %zu\\n", sizeof({struct}));')
        for field, _ in mirror._fields_:
            lines.append(f'  printf("{struct}.{field} %zu\\n", offsetof({struct}, {field}));')
    lines.append("  return 0; }")
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-o", str(exe), str(src)], check=True)
    c_layout = dict(line.rsplit(" ", 1) for line in subprocess.run([str(exe)], capture_output=True, text=True,
                                                                     check=True).stdout.splitlines())
    for struct in STRUCTS:
        mirror = getattr(native, MIRRORS[struct])
        assert int(c_layout[struct]) == ctypes.sizeof(mirror), struct
        for field, _ in mirror._fields_:
            assert int(c_layout[f"{struct}.{field}"]) == getattr(mirror, field).offset, f"{struct}.{field}"


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the behaviour without a GPU")
def test_calls_fail_loudly_without_gpu():
    from plm import native
    from plm.decoder import RoundDecoder
    from plm.model import PLMWeights, shape_config

    with pytest.raises(native.NativeError):
        native.Context()
    weights = PLMWeights.random(shape_config("plm-tiny", vocab=512, aux_vocab=64), seed=0, device="cpu")
    with pytest.raises(native.NativeError):
        RoundDecoder(weights, 4)
    buf = ctypes.create_string_buffer(256)
    native.library().plm_last_error(buf, 256)
    assert buf.value  # the failure left a message
    # entry points that take a context reject a missing one before touching a device
    desc = native.IcdfDesc(n_rows=1, vocab=8, top_k=4)
    assert native.library().plm_icdf_decode(None, ctypes.byref(desc), None) != 0
