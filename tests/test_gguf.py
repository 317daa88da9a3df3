"""The GGUF weight source against the reference's own reader (no GPU).

Every file is read twice: by vibeblade_b200.gguf (libvbq's reader) and by the reference's
vibeblade::GGUFFile (cpp/src/gguf.cpp, compiled from its sources into oracle/_ref with a
C shim).  Tensor tables, tensor bytes, every metadata accessor and every error message must
agree.  Files come from tests/gguf_files.py, which writes the container the reference's own
test helper writes (tests/test_loader.py:35-118), including the cases its tests cover:
metadata-only files, all value types, malformed headers and truncation.
"""
from __future__ import annotations

import numpy as np
import pytest

import gguf_files as G
from vibeblade_b200 import formats as F
from vibeblade_b200.gguf import GGUFFile
from vibeblade_b200.quantize import quantize


@pytest.fixture(scope="module")
def ref():
    from oracle.oracle import load_ref_gguf
    r = load_ref_gguf()
    if r is None:
        pytest.skip("the reference's GGUF reader (oracle/_ref) is not available")
    return r


def _compare_file(ref, path, keys):
    """Open with both readers; compare everything they expose."""
    h, err = ref.open(path)
    assert err is None, err
    try:
        g = GGUFFile(path)
        assert g.version() == ref.lib.vbr_gguf_version(h)
        mine = [(t.name, t.n_dims, t.dims, t.type, t.offset, t.size) for t in g.tensors()]
        assert mine == ref.tensors(h)
        for name, *_ in mine:
            info = g.tensor_info(name)  # for a repeated name: the last tensor of that name
            a = g.tensor_data(name)
            b = ref.tensor_data(h, name, info.size)
            assert a is not None and bytes(a) == b
        assert g.tensor_info("no.such.tensor") is None and g.tensor_data("no.such.tensor") is None
        assert ref.lib.vbr_gguf_has_tensor(h, b"no.such.tensor") == 0
        for k in keys:
            kb = k.encode()
            assert g.meta_int(k, -7) == ref.lib.vbr_gguf_meta_int(h, kb, -7), k
            assert g.meta_float(k, -7.5) == ref.lib.vbr_gguf_meta_float(h, kb, -7.5), k
            assert g.meta_bool(k, True) == bool(ref.lib.vbr_gguf_meta_bool(h, kb, 1)), k
            assert g.meta_bool(k, False) == bool(ref.lib.vbr_gguf_meta_bool(h, kb, 0)), k
            assert g.meta_string(k) == ref.meta_string(h, k), k
            assert g.meta_int_array(k) == ref.meta_int_array(h, k), k
            assert g.meta_float_array(k) == ref.meta_float_array(h, k), k
            assert g.meta_string_array(k) == ref.meta_string_array(h, k), k
        g.close()
    finally:
        ref.close(h)


def test_reference_test_helper_file(ref, tmp_path):
    """The reference tests' default mock: two kv pairs, no tensors."""
    p = G.write(tmp_path / "model.gguf", [("general.architecture", G.STRING, "llama"),
                                         ("llama.context_length", G.U32, 2048)], [])
    _compare_file(ref, p, ["general.architecture", "llama.context_length", "missing"])
    with GGUFFile(p) as g:
        assert g.meta_string("general.architecture") == "llama"
        assert g.meta_int("llama.context_length") == 2048
        assert g.tensors() == []


ALL_KV = [
    ("u8", G.U8, 200), ("i8", G.I8, -100), ("u16", G.U16, 60000), ("i16", G.I16, -3),
    ("u32", G.U32, 4000000000), ("i32", G.I32, -123456), ("f32", G.F32, 0.1), ("bool_t", G.BOOL, True),
    ("bool_f", G.BOOL, False), ("str", G.STRING, "llama é中"), ("u64", G.U64, 2 ** 63 + 5),
    ("i64", G.I64, -2 ** 40), ("f64", G.F64, 1.0 / 3.0),
    ("a_str", G.ARRAY, (G.STRING, ["<s>", "</s>", "", "toké"])),
    ("a_u32", G.ARRAY, (G.U32, [1, 2, 4000000000])), ("a_i32", G.ARRAY, (G.I32, [-1, 7])),
    ("a_u64", G.ARRAY, (G.U64, [2 ** 50, 3])), ("a_i64", G.ARRAY, (G.I64, [-2 ** 50])),
    ("a_f32", G.ARRAY, (G.F32, [0.5, -2.25, 1e-30])), ("a_u8", G.ARRAY, (G.U8, [1, 2, 3])),
    ("a_f64", G.ARRAY, (G.F64, [1.5])), ("a_bool", G.ARRAY, (G.BOOL, [True, False])),
    ("a_i16", G.ARRAY, (G.I16, [5, 6])), ("a_empty", G.ARRAY, (G.F32, [])),
    ("dup", G.I32, 1), ("dup", G.STRING, "second"),  # one table per kind of value
]


def _weights(qtype, K, N, seed):
    rng = np.random.default_rng(seed)
    return quantize(rng.normal(0, 0.02, (K, N)).astype(np.float32), qtype).numpy()


def _tensors():
    rng = np.random.default_rng(0)
    return [
        G.weight_tensor("blk.0.attn_q.weight", _weights(F.GGML_TYPE_Q4_K, 8, 512, 1), 8, 512, F.GGML_TYPE_Q4_K),
        G.weight_tensor("blk.0.ffn_down.weight", _weights(F.GGML_TYPE_Q6_K, 6, 256, 2), 6, 256, F.GGML_TYPE_Q6_K),
        G.weight_tensor("blk.0.ffn_up.weight", _weights(F.GGML_TYPE_Q8_0, 5, 96, 3), 5, 96, F.GGML_TYPE_Q8_0),
        ("blk.0.attn_q.bias", (512,), F.GGML_TYPE_F32, rng.normal(0, 1, 512).astype(np.float32).tobytes()),
        ("token_embd.weight", (64, 10), F.GGML_TYPE_F16, rng.normal(0, 1, 640).astype(np.float16).tobytes()),
        ("three_d", (32, 2, 3), F.GGML_TYPE_Q8_0, bytes(6 * 34)),
        ("blk.0.attn_q.weight", (256, 1), F.GGML_TYPE_Q4_K, bytes(144)),  # a later name replaces
        ("empty", (0,), F.GGML_TYPE_F32, b""),
    ]


def test_all_value_types_and_tensors(ref, tmp_path):
    p = G.write(tmp_path / "all.gguf", ALL_KV, _tensors())
    _compare_file(ref, p, sorted({k for k, _, _ in ALL_KV} | {"missing"}))
    with GGUFFile(p) as g:
        assert g.meta_int("u32") == 4000000000 - 2 ** 32  # kept as a signed 32-bit value
        assert g.meta_int("u16", 9) == 9                  # 16-bit values are not kept
        assert g.meta_string("dup") == "second" and g.meta_int("dup") == 1  # one table per kind
        assert g.meta_int_array("a_u32") == [1, 2, 4000000000 - 2 ** 32]
        assert g.meta_float_array("a_f32")[1] == -2.25
        assert g.meta_int_array("a_u8") == []             # arrays of other types are skipped
        assert g.data_offset() % 32 == 0
        assert g.matrix_shape("blk.0.ffn_up.weight") == (5, 96, F.GGML_TYPE_Q8_0)


def _malformed(case: str) -> bytes:
    t1 = [G.weight_tensor("w", bytes(144 * 2), 2, 256, F.GGML_TYPE_Q4_K)]
    kv = [("general.architecture", G.STRING, "llama")]
    full = G.build(kv, t1)
    wpos = full.index(b"w", 40)  # the tensor name in the table
    if case == "bad_magic":
        return G.build(kv, t1, magic=0x12345678)
    if case == "version":
        return G.build(kv, t1, version=4)
    if case == "small":
        return full[:20]
    if case == "implausible":
        return G.build(kv, t1, n_kv=2_000_000)
    if case == "str_len":
        return full[:24 + 4]
    if case == "str_data":
        return full[:24 + 8 + 5]
    if case == "meta_type":  # one key whose value type id is 13
        b = G.build([], t1, n_kv=1)
        return b[:24] + G.enc_str("k") + (13).to_bytes(4, "little") + b[24:]
    if case == "dims":
        return G.build(kv, [("w", (1, 1, 1, 1, 1), F.GGML_TYPE_F32, bytes(4))])
    if case == "dims_eof":
        return full[:wpos + 1 + 4 + 3]
    if case == "info_eof":
        return full[:wpos + 1 + 4 + 16 + 5]
    if case == "data_start":
        return full[:wpos + 1 + 4 + 16 + 12 + 1]
    if case == "value_eof":
        return G.build([("x", G.U64, 5)], [])[:-3]
    assert case == "array_eof"
    return G.build([("x", G.ARRAY, (G.F32, [1.0] * 10))], [])[:-8]


@pytest.mark.parametrize("case", ["bad_magic", "version", "small", "implausible", "str_len", "str_data",
                                  "meta_type", "dims", "dims_eof", "info_eof", "data_start", "value_eof",
                                  "array_eof"])
def test_malformed_files_fail_like_the_reference(ref, tmp_path, case):
    p = tmp_path / f"{case}.gguf"
    p.write_bytes(_malformed(case))
    _, err = ref.open(str(p))
    assert err is not None
    with pytest.raises(RuntimeError) as e:
        GGUFFile(str(p))
    if case == "array_eof":
        # Documented reference defect: its integer and float array loops
        # (cpp/src/gguf.cpp:116-138) read elements without a bounds check, so a cut-off
        # array reads past the file's buffer and the error only comes at the data section.
        # This reader stops at the array itself.
        assert err == "GGUF: data section starts past end of file"
        assert str(e.value).startswith("GGUF: read past end of file at offset ")
    else:
        assert str(e.value) == err


def test_tensor_data_past_end_fails_like_the_reference(ref, tmp_path):
    t = [("w", (256, 2), F.GGML_TYPE_Q4_K, bytes(144 * 2)), ("v", (32,), F.GGML_TYPE_F32, bytes(128))]
    b = G.build([], t, offsets=[0, 4096])[:-200]  # v's data is cut off
    p = tmp_path / "cut.gguf"
    p.write_bytes(b)
    h, err = ref.open(str(p))
    assert err is None
    try:
        ref_msg = ref.tensor_data(h, "v", 128)
        assert isinstance(ref_msg, str)
        with GGUFFile(str(p)) as g:
            assert bytes(g.tensor_data("w")) == bytes(144 * 2)
            with pytest.raises(RuntimeError) as e:
                g.tensor_data("v")
            assert str(e.value) == ref_msg
    finally:
        ref.close(h)


def test_missing_file_message(tmp_path):
    with pytest.raises(RuntimeError, match="Cannot open GGUF: "):
        GGUFFile(str(tmp_path / "nope.gguf"))


def test_tensor_data_keeps_the_file_alive(tmp_path):
    w = _weights(F.GGML_TYPE_Q4_K, 4, 256, 9)
    p = G.write(tmp_path / "a.gguf", [], [G.weight_tensor("w", w, 4, 256, F.GGML_TYPE_Q4_K)])
    a = GGUFFile(p).tensor_data("w")  # the file object goes away; the array keeps it
    assert np.array_equal(a, w.reshape(-1))


def test_dequant_row_errors_need_no_gpu(tmp_path):
    """VibeBladeFast.dequant_row's errors (cpp/src/bindings.cpp:407-436) come before any
    device work: an unknown tensor, a type outside its switch, and (here, where the
    reference would read past the tensor) a row beyond the tensor."""
    w = _weights(F.GGML_TYPE_Q4_K, 4, 256, 9)
    q2 = np.zeros((2, 84), np.uint8)  # Q2_K: read by dequantize, not by dequant_row
    p = G.write(tmp_path / "d.gguf", [], [G.weight_tensor("w", w, 4, 256, F.GGML_TYPE_Q4_K),
                                          G.weight_tensor("q2", q2, 2, 256, F.GGML_TYPE_Q2_K)])
    with GGUFFile(p) as f:
        with pytest.raises(RuntimeError, match="Tensor not found: nope"):
            f.dequant_row("nope")
        with pytest.raises(RuntimeError, match="Unsupported type for dequant_row"):
            f.dequant_row("q2")
        with pytest.raises(RuntimeError, match="runs past"):
            f.dequant_row("w", 4)
        with pytest.raises(RuntimeError, match="runs past"):
            f.dequant_row("w", 3, 512)
