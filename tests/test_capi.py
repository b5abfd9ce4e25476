"""The C ABI without a GPU: the library loads, exports every symbol include/ulm_b200.h declares,
the Python binding covers them, and argument validation fails with a message before any device
work. Also the model.bin v1 format round trip."""
import ctypes
import os
import re
import struct

import pytest
import torch

import unifiedlm_c_b200._lib as L
from unifiedlm_c_b200 import export

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "ulm_b200.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(ulm_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_functions():
    names = declared_functions()
    assert "ulm_memory_fwd" in names and "ulm_memory_bwd" in names and len(names) >= 10


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(L.LIB_PATH)
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing


def test_binding_covers_header():
    assert sorted(L.SIGNATURES) == declared_functions()


def _ctype_of(decl):
    """The ctypes type a C parameter or return declaration binds to."""
    decl = re.sub(r"\b(const|restrict)\b", " ", decl).strip()
    base = decl.replace("*", " ").split()[0]
    if "*" in decl:
        return ctypes.c_char_p if base == "char" else "ptr"
    return {"int": ctypes.c_int, "int64_t": ctypes.c_int64, "float": ctypes.c_float, "void": None}[base]


def declared_prototypes():
    """name -> (return type, [parameter types]) parsed from the header's prototypes."""
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    protos = {}
    for m in re.finditer(r"([A-Za-z_][A-Za-z0-9_ \*]*?)\b(ulm_[a-z0-9_]+)\s*\(([^)]*)\)\s*;", text):
        ret, name, params = m.group(1), m.group(2), m.group(3).strip()
        args = [] if params in ("", "void") else [_ctype_of(p_) for p_ in params.split(",")]
        protos[name] = (_ctype_of(ret), args)
    return protos


def test_binding_argument_types_match_header():
    """Every ctypes argtypes / restype in the binding agrees with the prototype in the header (count
    and kind of each parameter), so no call passes a mistyped or shifted argument."""
    protos = declared_prototypes()
    assert sorted(protos) == declared_functions()
    for name, (res, args) in L.SIGNATURES.items():
        want_res, want_args = protos[name]
        got_args = ["ptr" if a is ctypes.c_void_p or (isinstance(a, type) and issubclass(a, ctypes._Pointer))
                    else a for a in args]
        assert len(got_args) == len(want_args), (name, len(got_args), len(want_args))
        for i, (g, w) in enumerate(zip(got_args, want_args)):
            assert g == w, (name, i, g, w)
        assert (res if res is not None else None) == want_res, (name, res, want_res)


def test_version_and_helpers():
    lib = L.lib()
    assert lib.ulm_version() >= 1
    assert lib.ulm_operand_ld(13) == 16 and lib.ulm_operand_ld(64) == 64
    assert lib.ulm_memory_stats_bwd_scratch(2, 100, 70) >= 2 * 70 * 4 + 2 * 3 * 8


def test_validation_rejects_bad_arguments_without_device_work():
    lib = L.lib()
    dummy = ctypes.c_void_p(16)
    # bad precision code
    rc = lib.ulm_decayed_scores(dummy, 64, dummy, 64, dummy, 64, dummy, 1, 64, 64, 7, None)
    assert rc == L.ULM_ERR_INVALID and b"prec" in lib.ulm_last_error()
    # row stride shorter than the row
    rc = lib.ulm_memory_stats_fwd(dummy, dummy, dummy, dummy, dummy, dummy, dummy, L.ULM_BF16, 8, 1, 4, 16, None)
    assert rc == L.ULM_ERR_INVALID and b"ld_op" in lib.ulm_last_error()
    # null pointers
    rc = lib.ulm_memory_fwd(None, None, None, L.ULM_F32, None, None, None, None, None, None, None, None, None,
                            1, 4, 8, 8, L.ULM_PREC_BF16, None)
    assert rc == L.ULM_ERR_INVALID and b"null" in lib.ulm_last_error()
    # the unnormalised address form without its work buffer
    rc = lib.ulm_address_fwd(dummy, L.ULM_F32, dummy, 4, dummy, 64, dummy, dummy, dummy, dummy, 0, None, dummy, 64,
                             1, 8, 64, 64, L.ULM_PREC_BF16, None)
    assert rc == L.ULM_ERR_INVALID and b"work" in lib.ulm_last_error()
    # bad dtype
    rc = lib.ulm_causal_apply(dummy, 64, dummy, 64, dummy, 64, 5, 0, 1, 64, 64, L.ULM_PREC_BF16, None)
    assert rc == L.ULM_ERR_INVALID


def test_check_raises_with_message():
    lib = L.lib()
    rc = lib.ulm_decayed_scores(None, 1, None, 1, None, 1, None, 1, 1, 1, 9, None)
    with pytest.raises(L.UlmError, match="prec"):
        L.check(rc)


def test_cpu_tensors_are_refused():
    from unifiedlm_c_b200.kernel import unified_memory
    r = torch.rand(1, 8, 4)
    with pytest.raises(RuntimeError, match="CUDA"):
        unified_memory(r, torch.rand(1, 8, 4), torch.tensor(-0.1), torch.ones(4))


def test_model_bin_roundtrip(tmp_path, golden_dir):
    f = torch.load(os.path.join(golden_dir, "runc_tiny.pt"), weights_only=False)
    sd = f["state_dict"]
    path = tmp_path / "m.bin"
    export.write_model_bin(sd, str(path), f["max_seq_len"])
    raw = open(path, "rb").read()
    magic, version, dim, nl, hid, vocab, seq, conv, shared = struct.unpack_from("<Ii7i", raw, 0)
    # the fixture's classifier is untied from the embedding, so it is written after the final norm
    assert (magic, version, dim, nl, hid, vocab, seq, conv, shared) == (0x554C4D65, 1, 32, 2, 48, 512, 64, 4, 0)
    cfg, t = export.read_model_bin(str(path))
    assert cfg["dim"] == 32 and cfg["n_layers"] == 2
    assert torch.equal(t["layers.1.key.weight"], sd["layers.1.key.weight"].float())
    assert torch.equal(t["layers.0.conv"], sd["layers.0.conv.weight"][:, 0, :].float())
    lam = torch.exp(-torch.exp(sd["layers.0.log_rate"])).float()
    assert torch.equal(t["layers.0.lam"], lam.reshape(1))
    assert torch.equal(t["output.weight"], sd["output.weight"].float())
    expect = 256 + 4 * (512 * 32 + 2 * (32 + 32 * 4 + 48 * 32 + 48 + 32 * 48 + 32 * 32 + 48 + 2) + 32 + 512 * 32)
    assert len(raw) == expect
