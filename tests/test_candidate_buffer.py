"""Shard-wise candidate buffers against the reference's rank-0 fill and broadcast (CPU)."""
import numpy as np
import pytest
import torch

from oracle import opus_oracle as orc
from opus_b200.train.candidate_buffer import ShardedCandidateStream, read_header, write_shard


def make_files(tmp_path, sizes, token_bytes=2, seed=0, vocab=50257):
    rng = np.random.default_rng(seed)
    files, payloads = [], []
    for i, n in enumerate(sizes):
        toks = rng.integers(0, vocab, n)
        p = tmp_path / f"shard_{i:03d}.bin"
        write_shard(p, toks, token_bytes=token_bytes, eod=50256)
        files.append(p)
        payloads.append(toks)
    return files, payloads


@pytest.mark.parametrize("sizes,token_bytes,world,buffer_size,seq_len", [
    ([5000, 3000, 7000], 2, 4, 1024, 256),     # buffers cross file ends and wrap around the cycle
    ([2049, 2049], 4, 2, 1024, 512),           # int32 payload; a buffer ends exactly at a file end
    ([100, 0, 900, 4000], 2, 3, 300, 100),     # an empty file; more buffers than one cycle
    ([10000], 2, 8, 768, 256),                 # one file, eight ranks
])
def test_each_rank_reads_the_reference_slice(tmp_path, sizes, token_bytes, world, buffer_size, seq_len):
    files, payloads = make_files(tmp_path, sizes, token_bytes)
    n_buf = 9
    want = orc.candidate_buffers(payloads, buffer_size, world, n_buf)
    streams = [ShardedCandidateStream(files, buffer_size, seq_len, rank=r, world=world) for r in range(world)]
    for i in range(n_buf):
        for r, st in enumerate(streams):
            inputs, targets = st.next_buffer(device=None, pin=False)
            sl = want[i][r]
            n = buffer_size // seq_len
            np.testing.assert_array_equal(inputs.numpy(), sl[:-1][:n * seq_len].reshape(n, seq_len))
            np.testing.assert_array_equal(targets.numpy(), sl[1:][:n * seq_len].reshape(n, seq_len).astype(np.int64))
            assert inputs.dtype == torch.int32 and targets.dtype == torch.int64


def test_header_checks(tmp_path):
    p = tmp_path / "bad.bin"
    hdr = np.zeros(256, np.int32)
    hdr[0] = 1234
    p.write_bytes(hdr.tobytes())
    with pytest.raises(AssertionError, match="magic"):
        read_header(p)
    hdr[0], hdr[1] = 20240520, 2
    p.write_bytes(hdr.tobytes())
    with pytest.raises(AssertionError, match="version"):
        read_header(p)
    hdr[1], hdr[2], hdr[3] = 1, 10, 2
    p.write_bytes(hdr.tobytes() + np.zeros(5, np.uint16).tobytes())
    with pytest.raises(AssertionError, match="number of tokens"):
        read_header(p)
    files, _ = make_files(tmp_path, [300], token_bytes=2)
    assert read_header(files[0]) == (300, 2, 50256)
    with pytest.raises(ValueError):
        ShardedCandidateStream(files, 100, 256)


@pytest.mark.gpu
def test_buffer_lands_on_the_device(tmp_path):
    files, payloads = make_files(tmp_path, [6000, 5000])
    want = orc.candidate_buffers(payloads, 2048, 2, 3)
    st = ShardedCandidateStream(files, 2048, 1024, rank=1, world=2)
    for i in range(3):
        inputs, targets = st.next_buffer(device="cuda")
        assert inputs.is_cuda and targets.is_cuda
        np.testing.assert_array_equal(inputs.cpu().numpy().reshape(-1), want[i][1][:-1])
        np.testing.assert_array_equal(targets.cpu().numpy().reshape(-1), want[i][1][1:])
