"""GGUF checkpoints on the device.

The reference reads GGUF files with ``engine/gguf_parser.py:47-178``
(``GGUFFile``): mmap, parse the header, then decode or matvec tensors from
the mapping on every call.  ``DeviceGGUF`` parses the same format (v2/v3:
magic, version, tensor and key/value counts, typed metadata, tensor infos
with GGML dims stored innermost first, data section aligned to
``general.alignment``), uploads every tensor's raw GGUF bytes to the device
once through double-buffered pinned staging, and serves the ``GGUFFile``
surface the engine uses -- ``metadata``, ``tensors``, ``find``, ``tensor``,
``tensor_row``, ``tensor_bytes``, ``raw_tensor``, ``matvec``, ``matmul``,
``close`` and the context-manager protocol -- from device memory with this
package's kernels.  ``write_gguf`` writes such files (synthetic
checkpoints for tests and benchmarks).
"""
from __future__ import annotations

import mmap
import struct
from dataclasses import dataclass
from pathlib import Path

import numpy as np
import torch

from . import _lib, ops

MAGIC = b'GGUF'
# metadata value types of the GGUF format
U8, I8, U16, I16, U32, I32, F32, BOOL, STRING, ARRAY, U64, I64, F64 = range(13)
_FMT = {U8: 'B', I8: 'b', U16: 'H', I16: 'h', U32: 'I', I32: 'i', F32: 'f', BOOL: '?', U64: 'Q', I64: 'q', F64: 'd'}
# GGML tensor types: values per block, bytes per block
GGML_F32, GGML_F16 = 0, 1
BLOCK = {0: (1, 4), 1: (1, 2), 2: (32, 18), 8: (32, 34), 12: (256, 144), 13: (256, 176), 14: (256, 210)}


@dataclass
class TensorInfo:
    name: str
    shape: tuple          # logical shape, outermost first ([rows, cols] for matrices)
    ggml_type: int
    offset: int           # absolute byte offset in the file
    nbytes: int


def tensor_nbytes(ggml_type: int, shape) -> int:
    if ggml_type not in BLOCK:
        raise NotImplementedError(f'GGML type {ggml_type} is not supported')
    vals, nb = BLOCK[ggml_type]
    n = int(np.prod(shape, dtype=np.int64))
    if n % vals:
        raise ValueError(f'{n} values are not a whole number of {vals}-value blocks')
    return n // vals * nb


class _Reader:
    def __init__(self, buf):
        self.buf, self.pos = buf, 0

    def take(self, fmt):
        n = struct.calcsize('<' + fmt)
        if self.pos + n > len(self.buf):
            raise ValueError(f'truncated GGUF at byte {self.pos}')
        v = struct.unpack_from('<' + fmt, self.buf, self.pos)[0]
        self.pos += n
        return v

    def string(self):
        n = self.take('Q')
        if self.pos + n > len(self.buf):
            raise ValueError('truncated GGUF string')
        s = bytes(self.buf[self.pos:self.pos + n]).decode('utf-8', errors='replace')
        self.pos += n
        return s

    def value(self, t):
        if t == STRING:
            return self.string()
        if t == ARRAY:
            et, n = self.take('I'), self.take('Q')
            if n > 100_000_000:
                raise ValueError('unreasonable GGUF array length')
            return [self.value(et) for _ in range(n)]
        if t not in _FMT:
            raise ValueError(f'unsupported GGUF metadata value type {t}')
        return self.take(_FMT[t])


def parse_gguf(buf):
    """(version, metadata, {name: TensorInfo}, alignment) of a GGUF image
    (bytes, mmap or memoryview)."""
    r = _Reader(buf)
    if bytes(buf[:4]) != MAGIC:
        raise ValueError('not a GGUF file')
    r.pos = 4
    version = r.take('I')
    if version not in (2, 3):
        raise ValueError(f'GGUF version {version} unsupported; expected v2/v3')
    nt, nk = r.take('Q'), r.take('Q')
    if nt > 10_000_000 or nk > 1_000_000:
        raise ValueError('invalid GGUF counts')
    meta = {}
    for _ in range(nk):
        k = r.string()
        meta[k] = r.value(r.take('I'))
    align = int(meta.get('general.alignment', 32))
    if align <= 0 or align > 4096:
        align = 32
    infos = []
    for _ in range(nt):
        name = r.string()
        nd = r.take('I')
        if nd < 1 or nd > 8:
            raise ValueError(f'tensor {name}: invalid dimension count {nd}')
        dims = tuple(r.take('Q') for _ in range(nd))
        t, off = r.take('I'), r.take('Q')
        if any(d == 0 for d in dims):
            raise ValueError(f'tensor {name}: dimensions must be positive')
        if off % align:
            raise ValueError(f'tensor {name}: data offset {off} is not aligned to {align} bytes')
        infos.append((name, tuple(reversed(dims)), t, off))
    data_start = (r.pos + align - 1) // align * align
    tensors, seen = {}, set()
    for name, shape, t, off in infos:
        if name in seen:
            raise ValueError(f'duplicate tensor name {name!r}')
        seen.add(name)
        nbytes = tensor_nbytes(t, shape) if t in BLOCK else 0
        if data_start + off + nbytes > len(buf):
            raise ValueError(f'tensor {name} extends past the end of the file')
        tensors[name] = TensorInfo(name, shape, t, data_start + off, nbytes)
    spans = sorted((x.offset, x.offset + x.nbytes, x.name) for x in tensors.values() if x.nbytes)
    for a, b in zip(spans, spans[1:]):
        if b[0] < a[1]:
            raise ValueError(f'tensor data ranges overlap: {a[2]!r} and {b[2]!r}')
    return version, meta, tensors, align


def _kv_bytes(k, v):
    out = struct.pack('<Q', len(k.encode())) + k.encode()
    t, payload = _value_bytes(v)
    return out + struct.pack('<I', t) + payload


def _value_bytes(v):
    if isinstance(v, bool):
        return BOOL, struct.pack('<?', v)
    if isinstance(v, int):
        return (I32, struct.pack('<i', v)) if -2 ** 31 <= v < 2 ** 31 else (I64, struct.pack('<q', v))
    if isinstance(v, float):
        return F32, struct.pack('<f', v)
    if isinstance(v, str):
        b = v.encode()
        return STRING, struct.pack('<Q', len(b)) + b
    if isinstance(v, (list, tuple)):
        items = [_value_bytes(x) for x in v]
        et = items[0][0] if items else U32
        if any(t != et for t, _ in items):
            raise ValueError('GGUF arrays hold one element type')
        return ARRAY, struct.pack('<IQ', et, len(items)) + b''.join(p for _, p in items)
    raise ValueError(f'unsupported metadata value {v!r}')


def write_gguf(path, metadata: dict, tensors: dict, alignment: int = 32, version: int = 3):
    """Write a GGUF file.  ``tensors``: {name: (raw bytes, ggml_type, shape)}
    with shape outermost first ([rows, cols]); metadata values: int, float,
    bool, str or lists of one of those."""
    meta = dict(metadata)
    if alignment != 32:
        meta['general.alignment'] = alignment
    head = MAGIC + struct.pack('<IQQ', version, len(tensors), len(meta))
    head += b''.join(_kv_bytes(k, v) for k, v in meta.items())
    off, infos, blobs = 0, b'', []
    for name, (raw, t, shape) in tensors.items():
        raw = bytes(raw)
        if len(raw) != tensor_nbytes(t, shape):
            raise ValueError(f'{name}: {len(raw)} bytes for shape {shape} of type {t}')
        nb = name.encode()
        dims = tuple(reversed(shape))
        infos += struct.pack('<Q', len(nb)) + nb + struct.pack('<I', len(dims))
        infos += b''.join(struct.pack('<Q', d) for d in dims) + struct.pack('<IQ', t, off)
        blobs.append((off, raw))
        off = (off + len(raw) + alignment - 1) // alignment * alignment
    pre = head + infos
    data_start = (len(pre) + alignment - 1) // alignment * alignment
    with open(path, 'wb') as f:
        f.write(pre + b'\0' * (data_start - len(pre)))
        pos = 0
        for o, raw in blobs:
            f.write(b'\0' * (o - pos))
            f.write(raw)
            pos = o + len(raw)


class DeviceGGUF:
    """A GGUF file with every tensor's raw bytes resident on ``device``."""

    def __init__(self, path, device='cuda', names=None, chunk_bytes: int = 64 << 20):
        self.path = Path(path)
        self.device = torch.device(device)
        self._file = self.path.open('rb')
        self._map = mmap.mmap(self._file.fileno(), 0, access=mmap.ACCESS_READ)
        try:
            self.version, self.metadata, self.tensors, self.alignment = parse_gguf(self._map)
            self.device_tensors = {}
            self._upload([n for n in self.tensors if names is None or n in names], chunk_bytes)
        finally:
            self._map.close()
            self._file.close()
        self.lib = _lib.load()

    def _upload(self, names, chunk):
        """Copy file bytes -> pinned staging (two buffers) -> device, the host
        copy of one chunk overlapping the transfer of the previous one."""
        stage = [torch.empty(chunk, dtype=torch.uint8).pin_memory() for _ in range(2)]
        done = [None, None]
        s = torch.cuda.Stream(self.device)
        view = memoryview(self._map)
        k = 0
        for name in names:
            x = self.tensors[name]
            if x.nbytes == 0:
                continue
            dst = torch.empty(x.nbytes, dtype=torch.uint8, device=self.device)
            for a in range(0, x.nbytes, chunk):
                n = min(chunk, x.nbytes - a)
                b = k % 2
                if done[b] is not None:
                    done[b].synchronize()
                buf = stage[b]
                buf[:n].numpy()[:] = np.frombuffer(view[x.offset + a:x.offset + a + n], dtype=np.uint8)
                with torch.cuda.stream(s):
                    dst[a:a + n].copy_(buf[:n], non_blocking=True)
                    ev = torch.cuda.Event()
                    ev.record(s)
                done[b] = ev
                k += 1
            self.device_tensors[name] = dst
        s.synchronize()
        del view

    # -- the GGUFFile surface ---------------------------------------------
    def close(self):
        self.device_tensors.clear()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def find(self, *names):
        """The first of ``names`` present, else the first tensor whose name
        ends in '.' + one of them, tried in order (engine/gguf_parser.py:368-376:
        exact names before suffix matches, so that 'output.weight' never picks
        'blk.N.attn_output.weight'); None when nothing matches."""
        for n in names:
            if n in self.tensors:
                return n
        for n in names:
            for name in self.tensors:
                if name.endswith('.' + n):
                    return name
        return None

    def tensor_bytes(self, info) -> int:
        """Bytes of a tensor's raw GGUF data (engine/gguf_parser.py:147-152)."""
        return tensor_nbytes(info.ggml_type, info.shape)

    def raw_tensor(self, name) -> memoryview:
        """The tensor's raw GGUF bytes as host memory, like the reference's
        view into its mapping (engine/gguf_parser.py:153-156), copied back from
        the device."""
        return memoryview(self.device_tensors[name].cpu().numpy()).cast('B')

    def raw(self, name) -> torch.Tensor:
        """The tensor's raw GGUF bytes on the device (uint8)."""
        return self.device_tensors[name]

    def _rows_cols(self, name):
        x = self.tensors[name]
        if len(x.shape) != 2:
            raise ValueError(f'{name}: expected a matrix, got shape {x.shape}')
        return x.shape

    def tensor(self, name) -> np.ndarray:
        """Dequantised f32 values (engine/gguf_parser.py:170-174)."""
        x = self.tensors[name]
        return self.tensor_dev(name).cpu().numpy().reshape(x.shape)

    def tensor_dev(self, name) -> torch.Tensor:
        x = self.tensors[name]
        w = self.device_tensors[name]
        if x.ggml_type == GGML_F32:
            return w.view(torch.float32).reshape(x.shape)
        if x.ggml_type == GGML_F16:
            return w.view(torch.float16).float().reshape(x.shape)
        return ops.dequantize(w, x.ggml_type, x.shape)

    def tensor_row(self, name, row) -> np.ndarray:
        """One row of a matrix, dequantised (engine/gguf_parser.py:176-193)."""
        rows, cols = self._rows_cols(name)
        if not 0 <= int(row) < rows:
            raise IndexError(f'{name}: row {row} outside [0, {rows})')
        x = self.tensors[name]
        vals, nb = BLOCK[x.ggml_type]
        rb = cols // vals * nb
        w = self.device_tensors[name][int(row) * rb:(int(row) + 1) * rb]
        if x.ggml_type == GGML_F32:
            return w.view(torch.float32).cpu().numpy()
        if x.ggml_type == GGML_F16:
            return w.view(torch.float16).float().cpu().numpy()
        return ops.dequantize(w.contiguous(), x.ggml_type, (cols,)).cpu().numpy()

    def _mat(self, name, X):
        rows, cols = self._rows_cols(name)
        x = self.tensors[name]
        if X.shape[-1] != cols:
            raise ValueError(f'{name}: expected {cols} input columns, got {X.shape[-1]}')
        w = self.device_tensors[name]
        if x.ggml_type in (GGML_F32, GGML_F16):
            if X.shape[0] <= 16 and cols % 8 == 0 and w.data_ptr() % 16 == 0:
                # a few tokens (decode): the library's dense GEMV streams the f16/f32 rows once
                return ops.gemv(w, X.contiguous(), x.ggml_type, rows, cols)
            m = w.view(torch.float32 if x.ggml_type == GGML_F32 else torch.float16).reshape(rows, cols).float()
            return X @ m.T                      # prompt-sized batches: a plain library GEMM
        return ops.matmul(w, X, x.ggml_type, rows, cols)

    def _check_product(self, name, x_shape, batched, row_chunk):
        """The argument checks of engine/gguf_parser.py:187-197,297-307, with
        the reference's messages.  ``row_chunk`` bounds the reference's host
        memory per step; the device product has no such chunking, so it is
        only validated."""
        info = self.tensors[name]
        what = 'matmul' if batched else 'matvec'
        if len(info.shape) != 2:
            raise ValueError(f'{name}: {what} requires a 2-D tensor, got {info.shape}')
        cols = info.shape[1]
        if batched and (len(x_shape) != 2 or x_shape[1] != cols):
            raise ValueError(f'{name}: expected batch shape (tokens, {cols}), got {tuple(x_shape)}')
        if not batched and (len(x_shape) != 1 or x_shape[0] != cols):
            raise ValueError(f'{name}: expected vector shape ({cols},), got {tuple(x_shape)}')
        if row_chunk < 1:
            raise ValueError('row_chunk must be positive')

    def matvec(self, name, vector, *, row_chunk=1024):
        """W @ x (engine/gguf_parser.py:180-288): numpy in -> numpy out, CUDA
        tensor in -> CUDA tensor out."""
        if isinstance(vector, torch.Tensor):
            self._check_product(name, tuple(vector.shape), False, row_chunk)
            return self._mat(name, vector.float().reshape(1, -1)).reshape(-1)
        x = np.asarray(vector, dtype=np.float32)
        self._check_product(name, x.shape, False, row_chunk)
        x = torch.from_numpy(np.ascontiguousarray(x)).to(self.device).reshape(1, -1)
        return self._mat(name, x).reshape(-1).cpu().numpy()

    def matmul(self, name, vectors, *, row_chunk=1024):
        """X @ W^T for X [T, cols] (engine/gguf_parser.py:290-367)."""
        if isinstance(vectors, torch.Tensor):
            self._check_product(name, tuple(vectors.shape), True, row_chunk)
            return self._mat(name, vectors.float())
        x = np.asarray(vectors, dtype=np.float32)
        self._check_product(name, x.shape, True, row_chunk)
        x = torch.from_numpy(np.ascontiguousarray(x)).to(self.device)
        return self._mat(name, x).cpu().numpy()
