"""Host runtime (C++): HMAC-SHA256 against Python's hashlib/hmac, XOR parity repair,
file spill round trip, signed TCP tensor frames, page allocator."""
import hashlib
import hmac
import os
import threading

import pytest
import torch

from vramancer_b200 import runtime as rt


@pytest.mark.parametrize("n", [0, 1, 55, 56, 63, 64, 65, 1000, 1 << 20])
def test_sha256_and_hmac_match_python(n):
    data = os.urandom(n)
    assert rt.sha256(data) == hashlib.sha256(data).digest()
    for key in (b"", b"k", os.urandom(64), os.urandom(100)):
        tag = rt.sign(key, data)
        assert tag == hmac.new(key, data, hashlib.sha256).digest()
        assert rt.verify(key, data, tag)
        assert not rt.verify(key, data + b"x", tag)
    msgs = [os.urandom(i * 7) for i in range(10)]
    assert rt.sign_batch(b"key", msgs) == [hmac.new(b"key", m, hashlib.sha256).digest() for m in msgs]


def test_xor_parity_repairs_any_single_shard():
    shards = [os.urandom(4099) for _ in range(5)]
    par = rt.xor_parity(shards)
    for miss in range(5):
        got = rt.xor_repair([s if i != miss else None for i, s in enumerate(shards)], par)
        assert bytes(got) == shards[miss]
    big = [torch.randint(0, 255, (3 << 20,), dtype=torch.uint8) for _ in range(3)]
    p = rt.xor_parity(big, threads=4)
    assert bytes(rt.xor_repair([big[0], None, big[2]], p)) == big[1].numpy().tobytes()


def test_file_spill_round_trip(tmp_path):
    t = torch.randn(37, 129).to(torch.bfloat16)
    path = str(tmp_path / "spill.bin")
    n = rt.dump_tensor(path, t)
    assert n == t.numel() * 2
    out = torch.empty_like(t)
    rt.load_tensor(path, out)
    assert torch.equal(out, t)
    io = rt.AsyncFileIO(workers=2)
    bufs = [torch.randn(1000) for _ in range(4)]
    tickets = [io.write(str(tmp_path / f"a{i}.bin"), b) for i, b in enumerate(bufs)]
    assert all(io.wait(tk) == 4000 for tk in tickets)
    back = [torch.empty(1000) for _ in range(4)]
    tickets = [io.read(str(tmp_path / f"a{i}.bin"), b) for i, b in enumerate(back)]
    for tk in tickets:
        io.wait(tk)
    assert all(torch.equal(a, b) for a, b in zip(bufs, back))
    with pytest.raises(RuntimeError):
        rt.load_tensor(str(tmp_path / "spill.bin"), torch.empty(10 ** 6))   # short read


def _serve_once(listener, key, box):
    conn = listener.accept(10.0)
    try:
        box["got"] = rt.recv_tensors(conn, key)
    except Exception as e:  # noqa: BLE001 - the test inspects it
        box["err"] = e
    finally:
        conn.close()


@pytest.mark.parametrize("signed", [False, True])
def test_tcp_tensor_frames(signed):
    key = b"secret" if signed else b""
    lis = rt.listen("127.0.0.1", 0)
    box = {}
    th = threading.Thread(target=_serve_once, args=(lis, key, box))
    th.start()
    conn = rt.connect("127.0.0.1", lis.port)
    x = {"hidden": torch.randn(3, 64).to(torch.bfloat16), "ids": torch.arange(7), "empty": torch.empty(0)}
    rt.send_tensors(conn, x, {"step": 3}, key=key, chunk=1000)
    th.join(10)
    conn.close()
    lis.close()
    got, meta = box["got"]
    assert meta == {"step": 3}
    assert all(torch.equal(got[k], v) for k, v in x.items())


def test_tcp_frame_with_wrong_key_is_rejected():
    lis = rt.listen("127.0.0.1", 0)
    box = {}
    th = threading.Thread(target=_serve_once, args=(lis, b"right", box))
    th.start()
    conn = rt.connect("127.0.0.1", lis.port)
    rt.send_tensors(conn, {"a": torch.ones(100)}, key=b"wrong")
    th.join(10)
    conn.close()
    lis.close()
    assert "err" in box and "signature" in str(box["err"])


def test_page_allocator():
    pa = rt.page_allocator(8)
    a = pa.alloc(3)
    assert sorted(a) == [0, 1, 2] and pa.num_free == 5
    assert pa.alloc(6) == []                    # all-or-nothing
    pa.incref(a[0])
    assert not pa.decref(a[0]) and pa.refcount(a[0]) == 1
    pa.free_all(a)
    assert pa.num_free == 8
    with pytest.raises(ValueError):
        pa.decref(a[0])


def test_basic_tokenize_is_deterministic():
    out = rt.basic_tokenize(["hello, world", "hello"], 1000)
    assert len(out[0]) == 3 and out[0][0] == out[1][0]
    assert all(0 <= t < 1000 for t in out[0])


def test_tcp_frames_keep_every_dtype_aligned():
    lis = rt.listen("127.0.0.1", 0)
    box = {}
    th = threading.Thread(target=_serve_once, args=(lis, b"", box))
    th.start()
    conn = rt.connect("127.0.0.1", lis.port)
    x = {"a": torch.arange(3, dtype=torch.int32), "b": torch.arange(5, dtype=torch.int64),
         "c": torch.ones(3, dtype=torch.uint8), "d": torch.randn(2, 3, dtype=torch.float64)}
    rt.send_tensors(conn, x)
    th.join(10)
    conn.close()
    lis.close()
    got, _ = box["got"]
    assert all(torch.equal(got[k], v) for k, v in x.items())
