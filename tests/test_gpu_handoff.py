"""GPU: KV page hand-off through the C ABI (ubx_kv_pages_copy and the wire
header) against the reference's serialize/deserialize bytes (golden fixture)
and the oracle's gather/scatter. Every page byte is bit-exact; the checksum
equals the oracle's."""
import hashlib
import os

import numpy as np
import pytest
import torch

from conftest import HANDOFF_GOLDEN_NAMES, ROOT, sha

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def load_handoff(name, pkg):
    z = dict(np.load(os.path.join(ROOT, "tests", "golden", name + ".npz")))
    src = pkg.workloads.materialize_pool_host(int(z["seed"]), int(z["num_layers"]), int(z["num_blocks"]),
                                              int(z["block_size"]), int(z["num_kv_heads"]), int(z["head_dim"]),
                                              str(z["dtype"]))
    assert sha(src) == str(z["sha_src_pool"])
    return z, src


@pytest.mark.parametrize("name", HANDOFF_GOLDEN_NAMES)
def test_serialize_blocks_is_the_reference_payload(name, pkg, oracle):
    z, src = load_handoff(name, pkg)
    ho = pkg.handoff
    msg = ho.serialize_blocks(src.to(DEV), [int(p) for p in z["src_pages"]])
    h = ho.parse_header(msg)
    body = msg[64:]
    assert len(body) == int(z["payload_bytes"]) == h.payload_bytes
    assert hashlib.sha256(body).hexdigest() == str(z["sha_payload"])
    assert h.num_pages == len(z["src_pages"]) and h.dtype == 0 and h.num_layers == int(z["num_layers"])
    assert h.checksum == oracle.payload_checksum(body)


@pytest.mark.parametrize("name", HANDOFF_GOLDEN_NAMES)
def test_deserialize_blocks_matches_reference_pool(name, pkg):
    z, src = load_handoff(name, pkg)
    ho = pkg.handoff
    msg = ho.serialize_blocks(src.to(DEV), [int(p) for p in z["src_pages"]])
    dst = torch.zeros_like(src, device=DEV)
    ho.deserialize_blocks(dst, msg, [int(p) for p in z["dst_pages"]])
    torch.cuda.synchronize()
    pkg.check_device_errors()
    assert sha(dst.cpu()) == str(z["sha_dst_after"])


@pytest.mark.parametrize("dtype", ["bfloat16", "float16", "float32"])
def test_pack_unpack_roundtrip_vs_oracle(dtype, pkg, oracle):
    wl, ho = pkg.workloads, pkg.handoff
    seed = 40 + ["bfloat16", "float16", "float32"].index(dtype)
    src = wl.materialize_pool_host(seed, 4, 50, 16, 8, 112, dtype)
    dst0 = wl.materialize_pool_host(seed, 4, 40, 16, 8, 112, dtype, stream=31)
    sp = wl.portable_permutation(seed, 3, 50)[:23].tolist()
    dp = wl.portable_permutation(seed, 4, 40)[:23].tolist()
    ck = torch.zeros(1, dtype=torch.int64, device=DEV)
    payload = ho.pack_pages(src.to(DEV), sp, checksum=ck)
    ref_payload = oracle.gather_pages(src, sp)
    got = payload.cpu().view(-1).view(torch.uint8).numpy().tobytes()
    assert got == ref_payload
    assert (int(ck.item()) & (2 ** 64 - 1)) == oracle.payload_checksum(ref_payload)
    dst = dst0.to(DEV)
    ck2 = torch.zeros(1, dtype=torch.int64, device=DEV)
    ho.unpack_pages(payload, dst, dp, checksum=ck2)
    ref_dst = dst0.clone()
    oracle.scatter_pages(ref_payload, ref_dst, dp)
    torch.cuda.synchronize()
    assert torch.equal(dst.cpu(), ref_dst)
    assert int(ck2.item()) == int(ck.item())


@pytest.mark.parametrize("dtype", ["bfloat16", "float32"])
def test_transfer_pages_same_device(dtype, pkg, oracle):
    wl, ho = pkg.workloads, pkg.handoff
    src = wl.materialize_pool_host(50, 3, 30, 16, 8, 112, dtype)
    dst0 = wl.materialize_pool_host(51, 3, 33, 16, 8, 112, dtype, stream=31)
    sp, dp = [3, 17, 0, 29, 8], [32, 1, 5, 6, 20]
    dst = dst0.to(DEV)
    ho.transfer_pages(src.to(DEV), sp, dst, dp)
    ref = dst0.clone()
    oracle.scatter_pages(oracle.gather_pages(src, sp), ref, dp)
    torch.cuda.synchronize()
    assert torch.equal(dst.cpu(), ref)


def test_corrupted_message_and_wrong_pool_are_rejected(pkg):
    wl, ho = pkg.workloads, pkg.handoff
    src = wl.materialize_pool_host(60, 2, 10, 16, 8, 112, "bfloat16").to(DEV)
    msg = bytearray(ho.serialize_blocks(src, [1, 4, 7]))
    msg[64 + 1000] ^= 0x40  # one flipped bit in the payload, on the host
    dst = torch.zeros_like(src)
    with pytest.raises(RuntimeError, match="checksum"):
        ho.deserialize_blocks(dst, bytes(msg), [0, 2, 3])
    good = ho.serialize_blocks(src, [1, 4, 7])
    with pytest.raises(ValueError, match="dtype"):
        ho.deserialize_blocks(torch.zeros(src.shape, dtype=torch.float16, device=DEV), good, [0, 2, 3])
    with pytest.raises(ValueError):
        ho.deserialize_blocks(dst, good[:-2], [0, 2, 3])
    with pytest.raises(ValueError, match="pages"):
        ho.deserialize_blocks(dst, good, [0, 2])


def test_bad_page_flagged_not_faulted(pkg):
    wl, ho = pkg.workloads, pkg.handoff
    src = wl.materialize_pool_host(61, 2, 10, 16, 8, 112, "bfloat16").to(DEV)
    dst = torch.zeros_like(src)
    ho.transfer_pages(src, [1, 99, 2], dst, [0, 1, 2])
    with pytest.raises(RuntimeError, match="page id"):
        pkg.check_device_errors()
    torch.cuda.synchronize()
    assert torch.equal(dst[:, :, 0], src[:, :, 1]) and torch.equal(dst[:, :, 2], src[:, :, 2])
    assert not dst[:, :, 1].any()


def test_full_size_sequence_handoff_checksum(pkg):
    """A 2048-token prompt of the 24-layer 760M model (128 pages, 176 MB of K/V):
    pack on one pool, unpack into another at other page ids; the receiver's
    checksum of the bytes it scattered equals the sender's, and a sample of
    pages matches exactly."""
    ho = pkg.handoff
    g = torch.Generator(device=DEV)
    g.manual_seed(7)
    src = torch.randn((24, 2, 300, 16, 8, 112), generator=g, device=DEV).to(torch.bfloat16)
    dst = torch.zeros((24, 2, 400, 16, 8, 112), dtype=torch.bfloat16, device=DEV)
    sp = torch.randperm(300, generator=g, device=DEV)[:128]
    dp = torch.randperm(400, generator=g, device=DEV)[:128]
    c1 = torch.zeros(1, dtype=torch.int64, device=DEV)
    c2 = torch.zeros(1, dtype=torch.int64, device=DEV)
    payload = ho.pack_pages(src, sp, checksum=c1)
    ho.unpack_pages(payload, dst, dp, checksum=c2)
    torch.cuda.synchronize()
    assert int(c1.item()) == int(c2.item()) != 0
    for i in (0, 57, 127):
        assert torch.equal(dst[:, :, int(dp[i])], src[:, :, int(sp[i])])


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_transfer_pages_across_gpus_over_nvlink(pkg, oracle):
    wl, ho = pkg.workloads, pkg.handoff
    src_h = wl.materialize_pool_host(70, 3, 30, 16, 8, 112, "bfloat16")
    dst_h = wl.materialize_pool_host(71, 3, 20, 16, 8, 112, "bfloat16", stream=31)
    src, dst = src_h.to("cuda:0"), dst_h.to("cuda:1")
    sp, dp = [4, 9, 28, 0], [19, 3, 0, 7]
    ho.transfer_pages(src, sp, dst, dp)
    torch.cuda.synchronize("cuda:0")
    ref = dst_h.clone()
    oracle.scatter_pages(oracle.gather_pages(src_h, sp), ref, dp)
    assert torch.equal(dst.cpu(), ref)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_pull_pages_from_peer_gpu(pkg, oracle):
    """The decode worker's GPU runs the copy and reads the prefill pool on the
    other GPU (a peer source: plain loads over NVLink, no TMA load)."""
    wl, ho = pkg.workloads, pkg.handoff
    src_h = wl.materialize_pool_host(72, 3, 30, 16, 8, 112, "bfloat16")
    dst_h = wl.materialize_pool_host(73, 3, 20, 16, 8, 112, "bfloat16", stream=31)
    src, dst = src_h.to("cuda:0"), dst_h.to("cuda:1")
    sp, dp = [1, 29, 7, 12, 3], [0, 19, 4, 8, 11]
    ho.transfer_pages(src, sp, dst, dp, on="destination")
    torch.cuda.synchronize("cuda:1")
    ref = dst_h.clone()
    oracle.scatter_pages(oracle.gather_pages(src_h, sp), ref, dp)
    assert torch.equal(dst.cpu(), ref)
    with torch.cuda.device("cuda:1"):
        pkg.check_device_errors(torch.device("cuda:1"))


def _ipc_rank(rank, port, result_path):
    """Two worker processes, one GPU each (worker.py:47-51): the decode worker
    (rank 1) exports its pool over CUDA IPC, the prefill worker (rank 0) writes
    its pages straight into it with one kernel."""
    import sys
    sys.path.insert(0, ROOT)
    import torch.distributed as dist
    from __graft_entry__ import load_package
    from oracle import oracle
    pkg = load_package()
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=2)
    wl, ho = pkg.workloads, pkg.handoff
    src_h = wl.materialize_pool_host(80, 2, 24, 16, 8, 112, "bfloat16")
    dst_h = wl.materialize_pool_host(81, 2, 16, 16, 8, 112, "bfloat16", stream=31)
    sp, dp = [23, 5, 11], [2, 15, 9]
    token = [None]
    if rank == 1:
        dst = dst_h.to("cuda:1")
        torch.cuda.synchronize()
        token[0] = ho.ipc_export(dst)
    dist.broadcast_object_list(token, src=1)
    if rank == 0:
        m = ho.ipc_import(token[0], "cuda:0")
        ho.transfer_pages_to_ipc(src_h.to("cuda:0"), sp, m, tuple(dst_h.shape), dp)
        torch.cuda.synchronize()
    dist.barrier()  # the writes are complete before the owner reads
    if rank == 1:
        ref = dst_h.clone()
        oracle.scatter_pages(oracle.gather_pages(src_h, sp), ref, dp)
        with open(result_path, "w") as f:
            f.write("1" if torch.equal(dst.cpu(), ref) else "0")
    dist.barrier()
    if rank == 0:
        m.close()
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_ipc_handoff_between_worker_processes(tmp_path):
    import socket
    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    out = tmp_path / "ipc.txt"
    mp.start_processes(_ipc_rank, args=(port, str(out)), nprocs=2, join=True, start_method="spawn")
    assert out.read_text() == "1"
