"""The deployment loader's validation (exl3cu_model_open with
EXL3CU_MODEL_VALIDATE_ONLY: no GPU) against the reference reader's own test
(tests/test_model_reader.cpp of the reference) and against the restated
reader in oracle/model_reader.py, one corrupted field at a time.

Every case must give the oracle's verdict, and for a rejection the oracle's
message (the reference's wording, src/exl3_model.cpp:79-157)."""
import copy
import json
import struct

import numpy as np
import pytest

import model_dir as md


@pytest.fixture(scope="module")
def lib():
    from exl3_b200 import _lib

    return _lib.lib()


def _open(directory):
    """(ok, message, Exl3Model|None) from the B200 loader, validation only."""
    from exl3_b200 import Exl3InvalidArgument
    from exl3_b200.model import Exl3Model

    try:
        return True, "", Exl3Model(directory, validate_only=True)
    except Exl3InvalidArgument as e:
        return False, e.message, None


def _oracle(directory):
    from oracle.model_reader import ModelError, read_model

    try:
        return True, "", read_model(directory)
    except ModelError as e:
        return False, str(e), None


def _agree(directory):
    ok, msg, m = _open(directory)
    ook, omsg, info = _oracle(directory)
    assert ok == ook, (msg, omsg)
    if not ok:
        if omsg.startswith("JSON:"):
            assert msg.startswith("JSON:"), msg
        else:
            assert msg == omsg
    return ok, msg, m, info


def test_reference_reader_fixture(tmp_path):
    """tests/test_model_reader.cpp:37-43: tensor_count 4, payload 8708; then its four rejections (:64-72)."""
    d = md.reference_fixture()
    d.write(tmp_path)
    ok, _, m, info = _agree(tmp_path)
    assert ok
    assert m.tensor_count() == 4 and m.payload_bytes() == 8708
    assert m.hidden_size() == 128 and m.vocab_size() == 128
    assert m.bits_per_weight() == 8708 * 8 / 16384 == info.bits_per_weight
    assert [x.name for x in m.matrices()] == ["lm_head"] and m.head_name == "lm_head"
    assert m.matrices()[0].bits == 4 and m.matrices()[0].codebook == 2

    cases = []
    a = copy.deepcopy(d)
    a.manifest["reference_parameter_count"] = 1
    cases.append((a, "Model payload or budget mismatch"))
    b = copy.deepcopy(d)
    b.header_patch["lm_head.suh"] = {"data_offsets": [8190, 8446]}  # a valid span, overlapping the trellis
    cases.append((b, "Overlapping or missing tensor data"))
    c = copy.deepcopy(d)
    c.header_patch["lm_head.suh"] = {"shape": [-128]}
    cases.append((c, "Invalid dimension or offset"))
    e = copy.deepcopy(d)
    e.truncate = 1
    cases.append((e, "Invalid tensor data span"))
    for i, (dep, want) in enumerate(cases):
        dep.write(tmp_path / f"r{i}")
        ok, msg, _, _ = _agree(tmp_path / f"r{i}")
        assert not ok and msg == want, (i, msg)


def _mutations():
    """(label, fn(Deployment) -> Deployment or (Deployment, header_text)) one rule each."""
    muts = []

    def m(label):
        def deco(fn):
            muts.append((label, fn))
            return fn
        return deco

    @m("dtype U8")
    def _(d):
        d.header_patch["model.norm.weight"] = {"dtype": "U8"}

    @m("dtype not a string")
    def _(d):
        d.header_patch["model.norm.weight"] = {"dtype": 5}

    @m("zero dimension")
    def _(d):
        d.header_patch["model.norm.weight"] = {"shape": [0]}

    @m("real dimension")
    def _(d):
        d.header_patch["model.norm.weight"] = {"shape": [256.0]}

    @m("bool dimension")
    def _(d):
        d.header_patch["model.norm.weight"] = {"shape": [True]}

    @m("offsets triple")
    def _(d):
        d.header_patch["model.norm.weight"] = {"data_offsets": [0, 4, 8]}

    @m("offsets not an array")
    def _(d):
        d.header_patch["model.norm.weight"] = {"data_offsets": 4}

    @m("negative offset")
    def _(d):
        d.header_patch["model.norm.weight"] = {"data_offsets": [-4, 1020]}

    @m("end before begin")
    def _(d):
        h = d.header()["model.norm.weight"]["data_offsets"]
        d.header_patch["model.norm.weight"] = {"data_offsets": [h[1], h[0]]}

    @m("end past payload")
    def _(d):
        p = d.payload()
        d.header_patch["model.norm.weight"] = {"data_offsets": [p - 512, p + 512]}

    @m("length mismatch")
    def _(d):
        d.header_patch["model.norm.weight"] = {"shape": [255]}

    @m("missing dtype key")
    def _(d):
        d.header_patch["model.norm.weight"] = {"dtype": None}

    @m("gap between spans")
    def _(d):
        d.entries = [e for e in d.entries if e[0] != "model.layers.0.layer_types"] + [
            ("model.layers.0.layer_types", "I32", [3], np.array([1, 0, 2], np.int32).tobytes())]
        d.extra_payload = b"\0" * 4
        hdr = d.header()
        t = hdr["model.layers.0.layer_types"]["data_offsets"]
        d.header_patch["model.layers.0.layer_types"] = {"data_offsets": [t[0] + 4, t[1] + 4]}

    @m("trailing unaccounted bytes")
    def _(d):
        d.extra_payload = b"\0" * 16
        d.manifest["weight_payload_bytes"] = d.payload()

    @m("header length beyond file")
    def _(d):
        return d, "LEN"

    @m("manifest format")
    def _(d):
        d.manifest["format"] = "gguf"

    @m("manifest version 2")
    def _(d):
        d.manifest["version"] = 2

    @m("manifest version 1.0 (numeric equality holds)")
    def _(d):
        d.manifest["version"] = 1.0

    @m("manifest version string")
    def _(d):
        d.manifest["version"] = "1"

    @m("manifest kv_cache")
    def _(d):
        d.manifest["kv_cache"] = "q8_0"

    @m("manifest missing format")
    def _(d):
        del d.manifest["format"]

    @m("embedding type")
    def _(d):
        d.manifest["input_embedding"]["type"] = "separate"

    @m("embedding basis")
    def _(d):
        d.manifest["input_embedding"]["basis"] = "rotated"

    @m("embedding token axis")
    def _(d):
        d.manifest["input_embedding"]["token_axis"] = 0

    @m("hidden not a multiple of 128")
    def _(d):
        d.manifest["input_embedding"]["hidden_size"] = 200

    @m("vocab above 1048576")
    def _(d):
        d.manifest["input_embedding"]["vocab_size"] = 1048576 + 128

    @m("hidden zero")
    def _(d):
        d.manifest["input_embedding"]["hidden_size"] = 0

    @m("payload bytes mismatch")
    def _(d):
        d.manifest["weight_payload_bytes"] += 2

    @m("budget above 5 bpw")
    def _(d):
        d.manifest["reference_parameter_count"] = d.payload() * 8 // 5 - 1

    @m("budget just under 5 bpw passes")
    def _(d):
        d.manifest["reference_parameter_count"] = -(-d.payload() * 8 // 5)

    @m("parameter count as a real")
    def _(d):
        d.manifest["reference_parameter_count"] = float(d.manifest["reference_parameter_count"])

    @m("head source missing")
    def _(d):
        d.manifest["input_embedding"]["source"] = "output"

    @m("head source not a string")
    def _(d):
        d.manifest["input_embedding"]["source"] = 3

    @m("head geometry vs manifest")
    def _(d):
        d.manifest["input_embedding"]["vocab_size"] = 384

    @m("head trellis dtype")
    def _(d):
        d.header_patch["lm_head.trellis"] = {"dtype": "F16"}

    @m("head scale dtype")
    def _(d):
        d.header_patch["lm_head.svh"] = {"dtype": "I16"}

    @m("ambiguous head codebook")
    def _(d):
        d.entries.append(("lm_head.mcg", "I32", [], struct.pack("<I", md.MCG_MARKER)))
        d.manifest["weight_payload_bytes"] = d.payload()

    @m("wrong mul1 multiplier")
    def _(d):
        d.entries = [(n, t, s, struct.pack("<I", 0x12345678) if n == "lm_head.mul1" else b) for n, t, s, b in
                     d.entries]

    @m("wrong mcg multiplier")
    def _(d):
        d.entries = [(n, t, s, struct.pack("<I", 1) if n.endswith(".mcg") else b) for n, t, s, b in d.entries]

    @m("marker as F32")
    def _(d):
        d.header_patch["lm_head.mul1"] = {"dtype": "F32"}

    @m("matrix bits 9")
    def _(d):
        d.entries.append(("extra.trellis", "I16", [8, 8, 144], bytes(8 * 8 * 144 * 2)))
        d.manifest["weight_payload_bytes"] = d.payload()
        d.manifest["reference_parameter_count"] *= 2

    @m("matrix last dim not 16*bits")
    def _(d):
        d.entries.append(("extra.trellis", "I16", [8, 8, 40], bytes(8 * 8 * 40 * 2)))
        d.manifest["weight_payload_bytes"] = d.payload()
        d.manifest["reference_parameter_count"] *= 2

    @m("matrix not a multiple of 128")
    def _(d):
        d.entries.append(("extra.trellis", "I16", [4, 8, 64], bytes(4 * 8 * 64 * 2)))
        d.manifest["weight_payload_bytes"] = d.payload()
        d.manifest["reference_parameter_count"] *= 2

    @m("matrix without scales")
    def _(d):
        d.entries.append(("extra.trellis", "I16", [8, 8, 64], bytes(8 * 8 * 64 * 2)))
        d.manifest["weight_payload_bytes"] = d.payload()
        d.manifest["reference_parameter_count"] *= 2

    @m("exllamav3 embedding form is a plain tensor")
    def _(d):
        d.entries.append(("model.embed_tokens.trellis", "I16", [64, 130], bytes(64 * 130 * 2)))
        d.entries.append(("model.embed_tokens.signs", "F16", [2, 256], bytes(2 * 256 * 2)))
        d.manifest["weight_payload_bytes"] = d.payload()
        d.manifest["reference_parameter_count"] *= 2

    return muts


@pytest.mark.parametrize("label,fn", _mutations(), ids=[m[0] for m in _mutations()])
def test_rule_by_rule_against_oracle(tmp_path, label, fn):
    d = md.mixed_model()
    r = fn(d)
    header_text = None
    if isinstance(r, tuple):
        d, what = r
        if what == "LEN":
            text = json.dumps(d.header())
            d.write(tmp_path)
            blob = bytearray((tmp_path / "model.safetensors").read_bytes())
            blob[0:8] = struct.pack("<Q", len(blob))
            (tmp_path / "model.safetensors").write_bytes(bytes(blob))
            _agree(tmp_path)
            return
    d.write(tmp_path, header_text)
    _agree(tmp_path)


def test_mixed_model_inventory_matches_oracle(tmp_path):
    d = md.mixed_model()
    d.write(tmp_path)
    ok, _, m, info = _agree(tmp_path)
    assert ok
    assert m.tensor_count() == len(info.tensors) == len(d.entries)
    assert m.payload_bytes() == info.payload
    assert m.bits_per_weight() == info.bits_per_weight <= 5.0
    got = [(x.name, x.k, x.n, x.bits, x.codebook) for x in m.matrices()]
    want = [(x.name, x.k, x.n, x.bits, x.codebook) for x in info.matrices]
    assert got == want
    assert {x[3] for x in got} == {2, 3, 4, 6}  # mixed bit widths
    assert {x[4] for x in got} == {0, 1, 2}     # all three codebooks
    for t in m.tensors():
        o = info.tensors[t.name]
        assert (t.dtype, t.shape, t.nbytes) == (o.dtype, o.shape, o.end - o.begin)
        assert t.device_ptr == 0  # validate-only: nothing on a GPU
    assert [t.name for t in m.tensors()] == sorted(info.tensors)


def test_duplicate_header_key_is_rejected(tmp_path):
    """Stricter than nlohmann/json (which keeps the last duplicate): a repeated key is an error."""
    d = md.reference_fixture()
    text = json.dumps(d.header())
    dup = text[:-1] + ', "lm_head.suh": {"dtype": "F16", "shape": [128], "data_offsets": [8192, 8448]}}'
    d.write(tmp_path, dup)
    ok, msg, _ = _open(tmp_path)
    assert not ok and "duplicate key" in msg


@pytest.mark.parametrize("text,frag", [
    ('{"a": [' * 70 + ']' * 70 + '}', "nesting too deep"),
    ('{"a": 01}', "leading zero"),
    ('{"a": [1,]}', "invalid value"),
    ('{"a": "x\x01"}', "control character"),
    ('{"a": "\\ud800"}', "surrogate"),
    ('{"a": 1} x', "trailing characters"),
    ('{"a": tru}', "invalid literal"),
])
def test_json_reader_rejects_malformed_headers(tmp_path, text, frag):
    d = md.reference_fixture()
    d.write(tmp_path, text)
    ok, msg, _ = _open(tmp_path)
    assert not ok and msg.startswith("JSON:") and frag in msg, msg


def test_json_reader_accepts_escapes_and_metadata(tmp_path):
    d = md.reference_fixture()
    d.metadata = {"kéy": "v€\U0001f600 \"q\" \\ / \b\f\n\r\t", "n": [1, -2, 3.5e3, None, True, False]}
    d.write(tmp_path)
    ok, _, m, _ = _agree(tmp_path)
    assert ok and m.tensor_count() == 4


def test_missing_files(tmp_path):
    ok, msg, _, _ = _agree(tmp_path)
    assert not ok and msg == "Cannot open model weights"
    md.reference_fixture().write(tmp_path)
    (tmp_path / "hexagon-exl3.json").unlink()
    ok, msg, _, _ = _agree(tmp_path)
    assert not ok and msg == "Cannot open deployment manifest"
    (tmp_path / "model.safetensors").write_bytes(b"\0" * 7)
    ok, msg, _, _ = _agree(tmp_path)
    assert not ok and msg == "Invalid weight file size"


def test_open_arguments(lib, tmp_path):
    import ctypes

    from exl3_b200 import _lib

    h = ctypes.c_void_p()
    assert lib.exl3cu_model_open(None, 0, 1, ctypes.byref(h)) == _lib.INVALID_ARGUMENT
    md.reference_fixture().write(tmp_path)
    assert lib.exl3cu_model_open(str(tmp_path).encode(), 0, 4, ctypes.byref(h)) == _lib.INVALID_ARGUMENT
    assert b"flags" in lib.exl3cu_last_error()
    assert lib.exl3cu_model_open(str(tmp_path).encode(), 0, 1, ctypes.byref(h)) == 0
    out = (ctypes.c_uint16 * 128)()
    assert lib.exl3cu_model_embedding(h, 0, out) == _lib.NO_SUPPORT  # validate-only: no device copy
    assert lib.exl3cu_model_embedding(h, 128, out) == _lib.INVALID_ARGUMENT
    assert b"outside vocabulary" in lib.exl3cu_last_error()
    idx = ctypes.c_size_t()
    assert lib.exl3cu_model_find_matrix(h, b"nope", ctypes.byref(idx)) == _lib.INVALID_ARGUMENT
    assert lib.exl3cu_model_find_tensor(h, b"lm_head.suh", ctypes.byref(idx)) == 0
    assert lib.exl3cu_model_free(h) == 0
