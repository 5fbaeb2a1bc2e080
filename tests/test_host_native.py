"""The C++ host cores against their Python reference implementations."""
import random

import pytest

from lunaflux_b200.kv.page_allocator import (NativePageAllocator, OutOfPages, PageAllocatorError, PyPageAllocator,
                                             native_available)

pytestmark = pytest.mark.skipif(not native_available(), reason="host extension not built")


def test_allocator_differential_random():
    rng = random.Random(7)
    a = PyPageAllocator(24, max_generation=40)
    b = NativePageAllocator(24, max_generation=40)
    live = []
    for step in range(4000):
        op = rng.random()
        if op < 0.05 and a._ckpt is None:
            ta, tb = a.checkpoint(), b.checkpoint()
            n = rng.randint(0, min(3, a.free_page_count()))
            got = a.allocate_run(n)
            assert got == b.allocate_run(n)
            if rng.random() < 0.5:
                a.rollback_to(ta)
                b.rollback_to(tb)
            else:
                a.commit_checkpoint(ta)
                b.commit_checkpoint(tb)
                live.extend([p, 1, 0] for p in got)  # committed pages are owned now
        elif op < 0.35:
            n = rng.randint(1, 4)
            ea = eb = None
            try:
                ra = a.allocate_run(n)
            except OutOfPages:
                ea = True
            try:
                rb = b.allocate_run(n)
            except OutOfPages:
                eb = True
            assert ea == eb
            if not ea:
                assert ra == rb
                live.extend([p, 1, 0] for p in ra)
        elif live:
            e = rng.choice(live)
            kind = rng.choice(["ra", "rc", "xa", "xc"])
            try:
                if kind == "ra":
                    a.retain_active(e[0])
                    b.retain_active(e[0])
                    e[1] += 1
                elif kind == "rc":
                    a.retain_cached(e[0])
                    b.retain_cached(e[0])
                    e[2] += 1
                elif kind == "xa" and e[1]:
                    a.release_active(e[0])
                    b.release_active(e[0])
                    e[1] -= 1
                elif kind == "xc" and e[2]:
                    a.release_cached(e[0])
                    b.release_cached(e[0])
                    e[2] -= 1
            except PageAllocatorError:
                pytest.fail("unexpected allocator error")
            if e[1] == 0 and e[2] == 0:
                live.remove(e)
                assert not a.validate_active(e[0]) and not b.validate_active(e[0])
        assert (a.free_page_count(), a.allocated_page_count(), a.retired_page_count()) == \
            (b.free_page_count(), b.allocated_page_count(), b.retired_page_count())
        assert list(a._free) == list(b._free)
        b.debug_check_invariants()
    from lunaflux_b200.kv.page_allocator import PageId
    with pytest.raises(PageAllocatorError):
        b.release_active(PageId(10_000, 0))


def test_bpe_native_equals_reference():
    from lunaflux_b200.tokenizer.bpe import Tokenizer
    from .test_tokenizer import MERGES, make_json
    text, _ = make_json(MERGES + [("a", "a"), ("aa", "a"), ("e", "l")])
    tok = Tokenizer.from_json(text)
    assert tok._native is not None
    rng = random.Random(0)
    alphabet = b"unrelated aaaa el\x00\xc3\xa9"
    for _ in range(300):
        data = bytes(rng.choice(alphabet) for _ in range(rng.randint(0, 60)))
        assert tok._bpe(data) == tok._bpe_reference(data)


# ---------------------------------------------------------------- framed channel
import socket
import struct

from lunaflux_b200.engine import channel as chan


def _pair(native_a: bool, native_b: bool, frame_timeout_s: float = 0.3):
    a, b = socket.socketpair()
    ca = chan.open_channel(a.fileno(), 1 << 20, frame_timeout_s, native=native_a)
    cb = chan.open_channel(b.fileno(), 1 << 20, frame_timeout_s, native=native_b)
    return a, b, ca, cb


@pytest.mark.parametrize("na,nb", [(True, True), (True, False), (False, True), (False, False)])
def test_channel_roundtrip_across_implementations(na, nb):
    a, b, ca, cb = _pair(na, nb)
    msgs = [b"", b"x", bytes(range(256)) * 300]
    for m in msgs:
        ca.send(m, 1.0)
    for m in msgs:
        assert cb.recv(1.0) == m
    assert cb.recv(0.05) is None          # nothing pending: a timeout, not an error
    cb.send(b"back", 1.0)
    assert ca.recv(1.0) == b"back"


@pytest.mark.parametrize("native", [True, False])
def test_channel_rejects_corrupt_frames(native):
    closed = chan.CLOSED_ERRORS
    for bad in (struct.pack("<IIQ", 0xDEADBEEF, 1, chan.fnv1a64(b"a")) + b"a",       # magic
                struct.pack("<IIQ", chan.MAGIC, 1, chan.fnv1a64(b"a") ^ 1) + b"a",   # checksum
                struct.pack("<IIQ", chan.MAGIC, (1 << 20) + 1, 0)):                  # length
        a, b = socket.socketpair()
        c = chan.open_channel(b.fileno(), 1 << 20, 0.3, native=native)
        a.sendall(bad)
        with pytest.raises(closed):
            c.recv(1.0)
        with pytest.raises(closed):       # poisoned from now on
            c.recv(0.01)


@pytest.mark.parametrize("native", [True, False])
def test_channel_partial_frame_times_out_and_eof_is_closed(native):
    a, b = socket.socketpair()
    c = chan.open_channel(b.fileno(), 1 << 20, 0.2, native=native)
    a.sendall(struct.pack("<IIQ", chan.MAGIC, 10, 0) + b"abc")   # frame never completes
    with pytest.raises(chan.TIMEOUT_ERRORS):
        c.recv(1.0)
    a2, b2 = socket.socketpair()
    c2 = chan.open_channel(b2.fileno(), 1 << 20, 0.2, native=native)
    a2.close()
    with pytest.raises(chan.CLOSED_ERRORS):
        c2.recv(1.0)


def test_message_channel_carries_wire_frames():
    """Control messages cross the channel as binary worker-wire frames (no pickle)."""
    a, b = socket.socketpair()
    ma, mb = chan.MessageChannel(a), chan.MessageChannel(b)
    ma.send(("outs", 1, [(3, 7, False)], [], True))
    assert mb.recv(1.0) == ("outs", 1, [(3, 7, False)], [], True)
    ma.close()
    with pytest.raises(EOFError):
        mb.recv(1.0)


# ---------------------------------------------------------------- approved root
def test_approved_root_native_matches_reference(tmp_path):
    import os

    import numpy as np

    from lunaflux_b200.utils.approved_fs import ApprovedFsError, NativeApprovedRoot, PyApprovedRoot
    (tmp_path / "d").mkdir()
    (tmp_path / "d" / "w.bin").write_bytes(bytes(range(200)) * 50)
    (tmp_path / "outside.txt").write_text("secret")
    os.symlink(str(tmp_path / "outside.txt"), str(tmp_path / "d" / "link"))
    os.symlink(str(tmp_path / "d"), str(tmp_path / "dlink"))
    with PyApprovedRoot(str(tmp_path)) as p, NativeApprovedRoot(str(tmp_path)) as n:
        assert p.identity == n.identity
        dp, sp = p.read_snapshot("d/w.bin")
        dn, sn = n.read_snapshot("d/w.bin")
        assert dp == dn and sp == sn
        buf = np.zeros(20000, dtype=np.uint8)
        assert n.read_into("d/w.bin", buf) == sp
        assert bytes(buf[:10000]) == dp
        for loc in ("d/link", "dlink/w.bin", "../x", "/etc/passwd", "d/./w.bin", "d//w.bin", "", "d", "nope"):
            with pytest.raises(ApprovedFsError):
                p.read_snapshot(loc)
            with pytest.raises(ApprovedFsError):
                n.read_snapshot(loc)
        with pytest.raises(ApprovedFsError):
            n.read_snapshot("d/w.bin", 100)          # size limit
        with pytest.raises(ApprovedFsError):
            n.read_into("d/w.bin", np.zeros(10, dtype=np.uint8))
    with pytest.raises(ApprovedFsError):
        NativeApprovedRoot("relative/path")
