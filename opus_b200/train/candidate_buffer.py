"""Candidate buffers read shard-wise: every rank loads only its own tokens.

The reference's OPUS loader (train.py:1044-1097) has rank 0 read the next
buffer_size * world + 1 tokens of the training stream into host memory, copy
them to its GPU and broadcast them; every rank then keeps its slice
[rank * buffer_size, rank * buffer_size + buffer_size + 1).  The stream is the
training .bin files in cycle order (train.py:1038-1039), each a 256-int32
header (magic 20240520, version 1, token count, bytes per token 2 or 4, EOD
token id) followed by uint16 or int32 tokens (train.py:645-664).

Here each rank computes where its slice lies in the same stream from the
file headers alone and reads exactly those tokens from the files into pinned
memory, then copies them to its GPU: no rank-0 read of every rank's data and
no broadcast.  The tokens each rank ends up with are the reference's.
"""
from __future__ import annotations

import bisect
from pathlib import Path

import numpy as np
import torch

MAGIC = 20240520
HEADER_INTS = 256


def read_header(path) -> tuple[int, int, int]:
    """(token count, bytes per token, EOD token id or -1) of a .bin shard (train.py:645-658)."""
    header = np.fromfile(str(path), dtype=np.int32, count=HEADER_INTS)
    if header.size < 3 or int(header[0]) != MAGIC:
        raise AssertionError("magic number mismatch in the data .bin file")
    if int(header[1]) != 1:
        raise AssertionError("unsupported version")
    token_bytes = int(header[3]) if header.size > 3 else 2
    if token_bytes not in (2, 4):
        token_bytes = 2
    eod = int(header[4]) if header.size > 4 and int(header[4]) > 0 else -1
    n = int(header[2])
    payload = Path(path).stat().st_size - HEADER_INTS * 4
    if payload < n * token_bytes:
        raise AssertionError("number of tokens read does not match header")
    return n, token_bytes, eod


class ShardedCandidateStream:
    """The reference's candidate-buffer stream, each rank reading only its slice.

    files: the training shards in the order the reference cycles them.
    Buffer i covers global stream positions [i*(B*W+1), (i+1)*(B*W+1)) with
    B = buffer_size tokens per rank and W ranks; rank r keeps
    [r*B, r*B + B + 1) of it.
    """

    def __init__(self, files, buffer_size: int, seq_len: int, rank: int = 0, world: int = 1):
        self.files = [Path(f) for f in files]
        if not self.files:
            raise ValueError("no training files")
        if buffer_size < seq_len:
            raise ValueError(f"No sequences to process. Buffer size ({buffer_size}) may be smaller than seq_len "
                             f"({seq_len}).")
        self.buffer_size, self.seq_len, self.rank, self.world = int(buffer_size), int(seq_len), int(rank), int(world)
        self._meta = [read_header(f) for f in self.files]
        self.lengths = [m[0] for m in self._meta]
        if sum(self.lengths) == 0:
            raise ValueError("the training files hold no tokens")
        self.cum = np.concatenate([[0], np.cumsum(self.lengths)]).tolist()
        self.cycle = self.cum[-1]
        self.eod_token_id = next((m[2] for m in self._meta if m[2] > 0), -1)
        self._maps: dict[int, np.memmap] = {}
        self.position = 0  # global stream position of the next buffer

    def _payload(self, fi: int) -> np.memmap:
        mm = self._maps.get(fi)
        if mm is None:
            n, token_bytes, _ = self._meta[fi]
            dtype = np.uint16 if token_bytes == 2 else np.int32
            mm = np.memmap(self.files[fi], dtype=dtype, mode="r", offset=HEADER_INTS * 4, shape=(n,))
            self._maps[fi] = mm
        return mm

    def read(self, start: int, count: int, out: np.ndarray) -> None:
        """Stream positions [start, start+count) into out (int32), across files and cycles."""
        done = 0
        while done < count:
            g = (start + done) % self.cycle
            fi = bisect.bisect_right(self.cum, g) - 1
            off = g - self.cum[fi]
            take = min(count - done, self.lengths[fi] - off)
            out[done:done + take] = self._payload(fi)[off:off + take]
            done += take

    def next_buffer(self, device=None, pin: bool = True):
        """This rank's (inputs [n, seq_len] int32, targets [n, seq_len] int64) of the next buffer."""
        B = self.buffer_size
        mine = torch.empty(B + 1, dtype=torch.int32, pin_memory=pin and torch.cuda.is_available())
        self.read(self.position + self.rank * B, B + 1, mine.numpy())
        self.position += B * self.world + 1
        if device is not None:
            mine = mine.to(device, non_blocking=True)
        n = B // self.seq_len
        cut = n * self.seq_len
        inputs = mine[:-1][:cut].view(n, self.seq_len)
        targets = mine[1:][:cut].to(torch.int64).view(n, self.seq_len)
        return inputs, targets


def write_shard(path, tokens, token_bytes: int = 2, eod: int = 0) -> None:
    """A .bin shard in the reference's format (for tests and tooling)."""
    header = np.zeros(HEADER_INTS, dtype=np.int32)
    header[0], header[1], header[2], header[3], header[4] = MAGIC, 1, len(tokens), token_bytes, eod
    payload = np.asarray(tokens, dtype=np.uint16 if token_bytes == 2 else np.int32)
    with open(path, "wb") as f:
        f.write(header.tobytes())
        f.write(payload.tobytes())
