"""CPU: the KV hand-off (kvcache.py:268-277, worker.py:175-183 / :217-223).

* the oracle's gather / scatter reproduce the reference's serialize_blocks bytes
  and deserialize_blocks pool (golden fixture made by running them);
* the wire header's host functions (C ABI) accept good headers and reject bad
  ones before any device work;
* a two-rank exchange over gloo (prefill rank -> decode rank) carries a message
  whose header the receiver validates against its own pool, the payload landing
  at the receiver's page ids.
"""
import ctypes
import hashlib
import os

import numpy as np
import pytest
import torch

from conftest import HANDOFF_GOLDEN_NAMES, ROOT, sha


def load_handoff(name, pkg):
    z = dict(np.load(os.path.join(ROOT, "tests", "golden", name + ".npz")))
    src = pkg.workloads.materialize_pool_host(int(z["seed"]), int(z["num_layers"]), int(z["num_blocks"]),
                                              int(z["block_size"]), int(z["num_kv_heads"]), int(z["head_dim"]),
                                              str(z["dtype"]))
    assert sha(src) == str(z["sha_src_pool"])
    return z, src


@pytest.mark.parametrize("name", HANDOFF_GOLDEN_NAMES)
def test_oracle_matches_reference_serialize_deserialize(name, pkg, oracle):
    z, src = load_handoff(name, pkg)
    payload = oracle.gather_pages(src, z["src_pages"])
    assert len(payload) == int(z["payload_bytes"])
    assert hashlib.sha256(payload).hexdigest() == str(z["sha_payload"])
    dst = torch.zeros_like(src)
    oracle.scatter_pages(payload, dst, z["dst_pages"])
    assert sha(dst) == str(z["sha_dst_after"])


def test_checksum_known_answers(oracle):
    assert oracle.payload_checksum(b"") == 0
    words = np.array([1, 2, 3], dtype="<u4").tobytes()
    assert oracle.payload_checksum(words) == 1 * 1 + 2 * 3 + 3 * 5
    big = np.array([0xFFFFFFFF] * 4, dtype="<u4").tobytes()
    assert oracle.payload_checksum(big) == (0xFFFFFFFF * (1 + 3 + 5 + 7)) % 2 ** 64


def header(pkg, **kw):
    L = pkg.library
    h = L.KVWireHeader()
    args = dict(dtype=1, num_layers=24, num_kv_heads=8, head_dim=112, block_size=16, num_pages=5, checksum=123)
    args.update(kw)
    st = L.load().ubx_kv_wire_header_init(ctypes.byref(h), args["dtype"], args["num_layers"], args["num_kv_heads"],
                                          args["head_dim"], args["block_size"], args["num_pages"], args["checksum"])
    return st, h


def test_wire_header_roundtrip_and_rejections(pkg):
    L = pkg.library
    lib = L.load()
    st, h = header(pkg)
    assert st == 0
    raw = bytes(h)
    assert len(raw) == 64 and raw[:8] == b"UBXKVPG1"
    want = 24 * 2 * 5 * 16 * 8 * 112 * 2
    assert h.payload_bytes == want and h.checksum == 123 and h.version == 1
    h2 = L.KVWireHeader.from_buffer_copy(raw)
    assert lib.ubx_kv_wire_header_check(ctypes.byref(h2), 1, 24, 8, 112, 16, want) == 0
    # pool of another dtype / geometry: unsupported, no conversion
    assert lib.ubx_kv_wire_header_check(ctypes.byref(h2), 0, 24, 8, 112, 16, want) == L.ERR_UNSUPPORTED
    assert lib.ubx_kv_wire_header_check(ctypes.byref(h2), 1, 24, 4, 112, 16, want) == L.ERR_UNSUPPORTED
    # truncated payload, bad magic
    assert lib.ubx_kv_wire_header_check(ctypes.byref(h2), 1, 24, 8, 112, 16, want - 2) == L.ERR_INVALID_ARGUMENT
    bad = L.KVWireHeader.from_buffer_copy(b"XXXXXXXX" + raw[8:])
    assert lib.ubx_kv_wire_header_check(ctypes.byref(bad), 1, 24, 8, 112, 16, want) == L.ERR_INVALID_ARGUMENT
    assert header(pkg, dtype=9)[0] == L.ERR_INVALID_ARGUMENT


def test_page_copy_validation_before_launch(pkg):
    lib = pkg.library.load()
    E = pkg.library.ERR_INVALID_ARGUMENT
    # misaligned base
    assert lib.ubx_kv_pages_copy(8, 0, 0, 0, None, 0, 16, 0, 0, 0, None, 0, 1, 1, 64, 1, None, None, None) == E
    # packed side with strides other than the wire payload's
    assert lib.ubx_kv_pages_copy(16, 999, 64, 64, None, 0, 32, 128, 64, 64, None, 0, 1, 1, 64, 1, None, None,
                                 None) == E
    # no pages: nothing to do
    assert lib.ubx_kv_pages_copy(16, 0, 0, 0, None, 0, 32, 0, 0, 0, None, 0, 1, 0, 64, 1, None, None, None) == 0


def _rank_main(rank, world, port, result_path):
    import sys
    sys.path.insert(0, ROOT)
    import torch.distributed as dist
    from __graft_entry__ import load_package
    from oracle import oracle
    pkg = load_package()
    L = pkg.library
    lib = L.load()
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    z = dict(np.load(os.path.join(ROOT, "tests", "golden", "handoff_fp32.npz")))
    Ln, NB, KVH, D = int(z["num_layers"]), int(z["num_blocks"]), int(z["num_kv_heads"]), int(z["head_dim"])
    if rank == 0:  # prefill worker: header + payload, sent as one message
        src = pkg.workloads.materialize_pool_host(int(z["seed"]), Ln, NB, 16, KVH, D, "float32")
        payload = oracle.gather_pages(src, z["src_pages"])
        h = L.KVWireHeader()
        assert lib.ubx_kv_wire_header_init(ctypes.byref(h), 0, Ln, KVH, D, 16, len(z["src_pages"]),
                                           oracle.payload_checksum(payload)) == 0
        msg = torch.frombuffer(bytearray(bytes(h) + payload), dtype=torch.uint8)
        dist.send(torch.tensor([msg.numel()]), 1)
        dist.send(msg, 1)
    else:  # decode worker: validate against its own pool, place at its own pages
        n = torch.zeros(1, dtype=torch.int64)
        dist.recv(n, 0)
        msg = torch.empty(int(n.item()), dtype=torch.uint8)
        dist.recv(msg, 0)
        data = msg.numpy().tobytes()
        h = L.KVWireHeader.from_buffer_copy(data[:64])
        ok = lib.ubx_kv_wire_header_check(ctypes.byref(h), 0, Ln, KVH, D, 16, len(data) - 64) == 0
        ok = ok and oracle.payload_checksum(data[64:]) == h.checksum
        dst = torch.zeros((Ln, 2, NB, 16, KVH, D), dtype=torch.float32)
        oracle.scatter_pages(data[64:], dst, z["dst_pages"])
        with open(result_path, "w") as f:
            f.write(f"{int(ok)} {sha(dst)}")
    dist.barrier()
    dist.destroy_process_group()


def test_two_rank_handoff_protocol_gloo(tmp_path):
    import socket
    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    out = tmp_path / "rank1.txt"
    mp.start_processes(_rank_main, args=(2, port, str(out)), nprocs=2, join=True, start_method="spawn")
    ok, digest = out.read_text().split()
    z = dict(np.load(os.path.join(ROOT, "tests", "golden", "handoff_fp32.npz")))
    assert ok == "1" and digest == str(z["sha_dst_after"])


def test_invariant_divisor_identity():
    """The page-copy kernel divides by the page vector count and the page count
    with a multiply-high (Granlund & Montgomery 1994): with s = ceil(log2 d) and
    m = floor(2^32 (2^s - d) / d) + 1, n // d == (mulhi(n, m) + n) >> s for all
    32-bit n. Checked here for the divisors the kernel meets and edge values."""
    import random
    rng = random.Random(1)

    def magic(d):
        s = 0
        while (1 << s) < d:
            s += 1
        return ((1 << 32) * ((1 << s) - d)) // d + 1, s

    for d in [1, 2, 3, 7, 14, 112, 128, 1792, 1793, 4096, 65535, 123457, 2 ** 31 - 1, 2 ** 31, 2 ** 32 - 1]:
        m, s = magic(d)
        assert m < 2 ** 32
        for n in [0, 1, d - 1, d, d + 1, 2 ** 31 - 1, 2 ** 32 - 1] + [rng.getrandbits(32) for _ in range(5000)]:
            if 0 <= n < 2 ** 32:
                assert (((n * m) >> 32) + n) >> s == n // d, (d, n)


def test_transfer_direction_is_checked(pkg):
    """transfer_pages runs its kernel on the source (push) or the destination
    (pull) GPU; anything else is rejected before any device work."""
    import torch
    pool = torch.zeros((1, 2, 4, 16, 8, 112), dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="on must be"):
        pkg.handoff.transfer_pages(pool, [0], pool, [1], on="sideways")
