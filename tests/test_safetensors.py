"""The product's SafeTensors reader (needle_safetensors_*, the parser
needle_load uses) on the reference's own parser edge cases
(crates/needle-infer/tests/functional.rs:284-332, 474-497).  Host code only:
no GPU needed."""
import struct

import numpy as np
import pytest

from conftest import load_pkg

nb = load_pkg()


def st_bytes(header, data=b""):
    h = header.encode()
    return struct.pack("<Q", len(h)) + h + data


def test_unbalanced_brace_in_metadata_value():
    # functional.rs:284-301: the header's braces must not corrupt parsing
    st = nb.SafeTensors(st_bytes('{"__metadata__":{"k":"v"}}'))
    assert st.get_metadata("k") == "v"
    st = nb.SafeTensors(st_bytes('{"__metadata__":{"k":"v}}"}}'))
    assert st.get_metadata("k") == "v}}"


def test_escaped_quotes_in_metadata():
    # functional.rs:303-332: an escaped quote must not truncate the value
    st = nb.SafeTensors(st_bytes('{"__metadata__":{"key":"value with \\"quotes\\""}}'))
    val = st.get_metadata("key")
    assert val == 'value with "quotes"'
    assert st.get_metadata("absent") is None


def test_i4_shape_mismatch_returns_none():
    # functional.rs:474-497: 6 bytes = 12 nibbles cannot fill shape [4, 4]
    st = nb.SafeTensors(st_bytes('{"t":{"dtype":"I4","shape":[4,4],"data_offsets":[0,6]}}', b"\xab" * 6))
    assert st.get_f32("t") is None


def test_i4_and_bf16_decode():
    # safetensors.rs:83-119: BF16 widening and signed-nibble I4 (low nibble first)
    bf = np.array([1.5, -2.25], np.float32).view(np.uint32) >> 16
    hdr = ('{"a":{"dtype":"I4","shape":[2,2],"data_offsets":[0,2]},'
           '"b":{"dtype":"BF16","shape":[2],"data_offsets":[2,6]}}')
    st = nb.SafeTensors(st_bytes(hdr, bytes([0x7F, 0x18]) + bf.astype(np.uint16).tobytes()))
    assert st.get_f32("a").tolist() == [-1.0, 7.0, -8.0, 1.0]
    assert st.get_f32("b").tolist() == [1.5, -2.25]


@pytest.mark.parametrize("bad", [b"", b"\x01\x00", struct.pack("<Q", 100) + b"{}",
                                 st_bytes('{"t":{"dtype":"F32","shape":[1],"data_offsets":[0,8]}}', b"\0" * 4),
                                 st_bytes('{"t":{"dtype":"Q9","shape":[1],"data_offsets":[0,4]}}', b"\0" * 4),
                                 st_bytes('["not an object"]')])
def test_malformed_buffers_are_rejected(bad):
    with pytest.raises(nb.NeedleError):
        nb.SafeTensors(bad)
