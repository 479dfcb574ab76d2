"""The O2 Eshkol bridge's host-side behaviour (no GPU): argument checks,
builder lifecycle, the last-error category, and the state file format
(written atomically, read back bit for bit, corruption rejected)."""
import ctypes as C
import struct

import numpy as np
import pytest

import eshkol_transformer_b200 as etb
from o2_bridge import bind


@pytest.fixture(scope="module")
def br():
    return bind(etb.load())


def test_builder_arguments_and_errors(br):
    assert br.et_o2_private_builder_create_v1(0, 0, 0, 0, 0, 0, 0) is None
    assert br.et_o2_private_last_error_category_v1() == 1
    assert br.et_o2_private_builder_create_v1(2, 7, 0, 0, 0, 0, 0) is None  # unknown clip kind
    assert br.et_o2_private_builder_create_v1(2, 1, 0, 0, 0, 0, 0) is None  # clip bound 0
    b = br.et_o2_private_builder_create_v1(2, 0, 0, 0, 0, 0, 0)
    assert b is not None and br.et_o2_private_last_error_category_v1() == 0
    one = 0x3f800000
    ident = C.c_int(1)
    assert br.et_o2_private_builder_set_v1(b, 0, None, C.addressof(ident), 1, 1, 1, one, 0) == 1
    assert br.et_o2_private_builder_set_v1(b, 5, C.addressof(ident), C.addressof(ident),
                                           1, 1, 1, one, 0) == 1  # index outside the builder
    assert br.et_o2_private_builder_set_v1(b, 0, C.addressof(ident), C.addressof(ident),
                                           1, one, 1, one, 0) == 1  # beta1 = 1
    assert br.et_o2_private_builder_finish_v1(b) is None  # unbound slots
    assert br.et_o2_private_last_error_category_v1() == 7
    assert br.et_o2_private_builder_abort_v1(b) == 0
    assert br.et_o2_private_optimizer_step_v1(None) == 1
    assert br.et_o2_private_optimizer_completed_updates_v1(None) == -1


def _state_bytes(entries, completed=3):
    out = b"ETB2O2S\x01" + struct.pack("<IIIIQQQQ", 0, 0, 0, 0, 0, 0, completed, len(entries))
    for m, v, opts in entries:
        out += struct.pack("<Q", m.size) + struct.pack("<5I", *opts)
        out += m.astype(np.float32).tobytes() + v.astype(np.float32).tobytes()
    h = 0xcbf29ce484222325
    for byte in out:
        h = ((h ^ byte) * 0x100000001b3) & 0xffffffffffffffff
    return out + struct.pack("<Q", h)


def test_state_file_round_trip_and_corruption(br, tmp_path):
    rng = np.random.default_rng(5)
    opts = (0x3a83126f, 0x3f666666, 0x3f7fbe77, 0x322bcc77, 0x3c23d70a)
    entries = [(rng.standard_normal(n).astype(np.float32),
                np.abs(rng.standard_normal(n)).astype(np.float32), opts) for n in (7, 100)]
    blob = _state_bytes(entries)
    src = tmp_path / "in.state"
    src.write_bytes(blob)
    st = br.et_b200_o2_state_read_v1(str(src).encode())
    assert st is not None, br.et_b200_o2_bridge_last_error_message_v1()
    dst = tmp_path / "out.state"
    dst.write_bytes(b"an older file")
    assert br.et_b200_o2_state_write_v1(st, str(dst).encode()) == 0
    assert dst.read_bytes() == blob  # replaced in full, byte for byte
    assert not [p for p in tmp_path.iterdir() if ".tmp." in p.name]  # no temporary left
    assert br.et_o2_private_optimizer_state_release_v1(st) == 0
    for bad in (blob[:-1], blob[:40], blob[:60] + bytes([blob[60] ^ 1]) + blob[61:]):
        src.write_bytes(bad)
        assert br.et_b200_o2_state_read_v1(str(src).encode()) is None
        assert br.et_o2_private_last_error_category_v1() == 7
    assert br.et_b200_o2_state_read_v1(str(tmp_path / "missing").encode()) is None
