"""Safetensors header validation, one case per check (reference:
model/safetensors_reader/reader_test.mbt: length prefix, envelope, strict
JSON, duplicate keys, exact int64 numbers, tensor fields, byte ranges,
complete payload, tensor-count bound)."""
import struct

import pytest
import torch

from lunaflux_b200.models.safetensors import (ReaderLimits, SafetensorsError, SafetensorsFile, declared_header_bytes,
                                              parse_header, save_file)

LIM = ReaderLimits(max_header_bytes=4096, max_tensor_count=8, max_payload_bytes=4096)


def fixture(header: str, payload_bytes: int = 0) -> bytes:
    h = header.encode()
    return struct.pack("<Q", len(h)) + h + bytes(payload_bytes)


def with_length(header: str, declared: int) -> bytes:
    return struct.pack("<Q", declared) + header.encode()


def kind_of(buf: bytes, limits=LIM):
    with pytest.raises(SafetensorsError) as ei:
        parse_header(buf, len(buf), limits)
    return ei.value.kind, ei.value.entry


def W(dtype="BF16", shape="[2]", offs="[0,4]"):
    return '{"w":{"dtype":"%s","shape":%s,"data_offsets":%s}}' % (dtype, shape, offs)


def test_valid_header_keeps_payload_relative_ranges():
    buf = fixture('{"__metadata__":{"format":"pt"},"a":{"dtype":"F32","shape":[2],"data_offsets":[0,8]},'
                  '"b":{"dtype":"BF16","shape":[1,2],"data_offsets":[8,12]}}', 12)
    start, tensors, meta = parse_header(buf, len(buf), LIM)
    assert meta == {"format": "pt"}
    assert start == len(buf) - 12
    assert (tensors["a"].begin, tensors["a"].end, tensors["b"].shape) == (0, 8, (1, 2))


def test_length_prefix():
    assert declared_header_bytes(with_length("", 37), LIM) == 37
    with pytest.raises(SafetensorsError) as ei:
        declared_header_bytes(with_length("x", 1), LIM)        # prefix must be exactly 8 bytes
    assert ei.value.kind == "envelope"
    with pytest.raises(SafetensorsError) as ei:
        declared_header_bytes(with_length("", 4097), LIM)
    assert ei.value.kind == "header_too_large"
    assert kind_of(b"short")[0] == "missing_length"
    assert kind_of(with_length("{}", 1 << 63))[0] == "header_too_large"
    assert kind_of(with_length("{}", 2147483648))[0] == "header_too_large"
    assert kind_of(fixture("{}"), ReaderLimits(max_header_bytes=1))[0] == "header_too_large"
    assert kind_of(with_length("{}", 3))[0] == "truncated_header"


@pytest.mark.parametrize("buf,kind", [
    (fixture(" {}"), "envelope"),
    (fixture("{}\n"), "envelope"),
    (fixture('{"x":}'), "json"),
    (fixture("[]"), "envelope"),
    (fixture('{"__metadata__":[]}'), "metadata"),
    (fixture('{"__metadata__":{"format":1}}'), "metadata"),
    (bytes([2, 0, 0, 0, 0, 0, 0, 0]) + b"{\xff", "envelope"),
    (bytes([3, 0, 0, 0, 0, 0, 0, 0]) + b"{\xff}", "encoding"),
])
def test_envelope_encoding_json_and_metadata(buf, kind):
    assert kind_of(buf)[0] == kind


def test_space_padding_is_header_but_trailing_bytes_are_payload():
    parse_header(fixture("{}   "), len(fixture("{}   ")), LIM)
    # "{} " declared as 2 bytes: the space is payload no tensor covers
    assert kind_of(with_length("{} ", 2))[0] == "payload_mismatch"


@pytest.mark.parametrize("header", [
    '{"w":{"dtype":"BF16","shape":[1],"data_offsets":[0,2]},"w":{"dtype":"BF16","shape":[1],"data_offsets":[0,2]}}',
    '{"w":{"dtype":"BF16","dtype":"F16","shape":[1],"data_offsets":[0,2]}}',
    '{"w":{"dtype":"BF16","sh\\u0061pe":[1],"shape":[1],"data_offsets":[0,2]}}',
])
def test_duplicate_names_and_fields(header):
    assert kind_of(fixture(header, 2))[0] == "json"


@pytest.mark.parametrize("header", [W(shape="[1.0]", offs="[0e0,2e0]"), W(shape="[1]", offs="[0,2]")])
def test_integral_json_numbers_are_exact_integers(header):
    buf = fixture(header, 2)
    _, t, _ = parse_header(buf, len(buf), LIM)
    assert t["w"].nbytes == 2 and t["w"].shape == (1,)


def test_int64_max_shape_reaches_size_validation():
    assert kind_of(fixture(W(shape="[9223372036854775807]", offs="[0,2]"), 2)) == ("size_overflow", 0)
    assert kind_of(fixture(W(shape="[4294967296, 4294967296]", offs="[0,2]"), 2)) == ("size_overflow", 0)


@pytest.mark.parametrize("header,kind", [
    ('{"w":[]}', "tensor_field"),
    ('{"w":{"shape":[2],"data_offsets":[0,4]}}', "tensor_field"),
    ('{"w":{"dtype":1,"shape":[2],"data_offsets":[0,4]}}', "tensor_field"),
    ('{"w":{"dtype":"BF16","shape":{},"data_offsets":[0,4]}}', "tensor_field"),
    (W(shape="[2.5]"), "integer"),
    (W(shape="[true]"), "integer"),
    (W(shape="[9223372036854775808]"), "integer"),
    (W(shape="[-2]"), "integer"),
    (W(offs="[0]"), "tensor_field"),
    ('{"w":{"dtype":"BF16","shape":[2],"data_offsets":[0,4],"extra":0}}', "tensor_field"),
    (W(dtype="Q4"), "dtype"),
    (W(shape="[1,1,1,1,1,1,1,1,2]"), "rank"),
    (W(offs="[-1,3]"), "byte_range"),
    (W(offs="[4,0]"), "byte_range"),
    (W(offs="[2,6]"), "outside_payload"),
    (W(offs="[0,2]"), "size_mismatch"),
    (W(dtype="F32"), "size_mismatch"),
    ('{"":{"dtype":"BF16","shape":[2],"data_offsets":[0,4]}}', "name"),
])
def test_tensor_entries(header, kind):
    assert kind_of(fixture(header, 4)) == (kind, 0)


def test_payload_must_be_tiled_exactly():
    assert kind_of(fixture(W(), 6))[0] == "payload_mismatch"              # trailing bytes
    hole = ('{"left":{"dtype":"BF16","shape":[1],"data_offsets":[0,2]},'
            '"right":{"dtype":"BF16","shape":[1],"data_offsets":[4,6]}}')
    assert kind_of(fixture(hole, 6))[0] == "payload_mismatch"
    overlap = ('{"a":{"dtype":"BF16","shape":[2],"data_offsets":[0,4]},'
               '"b":{"dtype":"BF16","shape":[2],"data_offsets":[2,6]}}')
    assert kind_of(fixture(overlap, 6))[0] == "overlap"
    # empty tensors take no bytes and may sit anywhere inside the payload
    ok = ('{"a":{"dtype":"BF16","shape":[2],"data_offsets":[0,4]},'
          '"e":{"dtype":"F32","shape":[0,3],"data_offsets":[4,4]}}')
    buf = fixture(ok, 4)
    assert parse_header(buf, len(buf), LIM)[1]["e"].nbytes == 0


def test_limits_checked_before_decoding():
    two = ('{"a":{"dtype":"BF16","shape":[1],"data_offsets":[0,2]},'
           '"b":{"dtype":"BF16","shape":[1],"data_offsets":[2,4]}}')
    assert kind_of(fixture(two, 4), ReaderLimits(max_tensor_count=1))[0] == "too_many_tensors"
    # the payload bound is checked before the malformed JSON is parsed
    assert kind_of(fixture('{"x":}', 5), ReaderLimits(max_payload_bytes=4))[0] == "outside_payload"
    assert kind_of(fixture('{"ww":{"dtype":"BF16","shape":[2],"data_offsets":[0,4]}}', 4),
                   ReaderLimits(max_name_length=1))[0] == "name"


def test_writer_output_passes_the_reader(tmp_path):
    t = {"x": torch.randn(3, 5), "y": torch.arange(7, dtype=torch.int32), "z": torch.empty(0, 4, dtype=torch.bfloat16)}
    p = str(tmp_path / "m.safetensors")
    save_file(t, p, {"format": "pt"})
    with SafetensorsFile(p) as f:
        for k, v in t.items():
            assert torch.equal(f.tensor(k), v)
