"""Serialise an :class:`IRGraph` into the flat blob the native engine parses.

Layout (all little-endian int64 unless noted; parsed by csrc/engine.cpp):

  header (12 words): magic "FTBGRAPH", version 1, n_nodes, input_id, output_id,
                     max_batch, flags, kernel_policy, static_batch,
                     n_weight_floats, nodes_offset, weights_offset
  nodes (20 words each): id, op, n_inputs, inputs[4], rank, dims[4],
                     stride_h, stride_w, pad_h, pad_w, dil_h, dil_w,
                     const_offset (floats), const_count
  weights: float32, each constant starting on a 64-byte boundary

Nodes not reachable from the output are dropped (for example a Linear weight
whose transposed copy replaced it) and ids are renumbered densely in
execution order.
"""

from __future__ import annotations

import hashlib
import struct
from typing import Dict, List

import numpy as np

from .frontend import OPS, IRGraph

MAGIC = b"FTBGRAPH"
VERSION = 1
HEADER_WORDS = 12
NODE_WORDS = 20

FLAG_DYNAMIC = 1
FLAG_FUSION = 2
FLAG_BIAS_FIRST_FUSED = 4
FLAG_NO_FOLD = 8  # reference fusion only (no epilogue folding, FLATTEN copies): reproduces the reference plan

# kernel policies (csrc/engine.hpp: KernelPolicy)
POLICIES = {"auto": 0, "simt": 1, "simt_exact": 2, "tcgen05": 3}


def _live_nodes(g: IRGraph) -> List[int]:
    keep = set()
    stack = [g.output_id, g.input_id]
    while stack:
        n = stack.pop()
        if n in keep:
            continue
        keep.add(n)
        stack.extend(g.nodes[n].inputs)
    return sorted(keep)


TUNE_MAGIC = b"FTBTUNE1"
TUNE_WORDS = 9  # step, batch_lo, batch_hi, family, tc_bn, tc_bk, tc_mh, tc_pair, fuse_head


def with_tuning(blob: bytes, records) -> bytes:
    """The blob with its tuning trailer replaced by ``records`` (none: removed).

    The trailer follows the weights at the next 8-byte boundary: the magic
    ``FTBTUNE1``, the record count and 9 little-endian int64 per record."""
    _, version, n_nodes = struct.unpack_from("<8sqq", blob, 0)
    n_w, _, w_off = struct.unpack_from("<3q", blob, 9 * 8)
    end = (w_off + n_w * 4 + 7) // 8 * 8
    out = bytearray(blob[:w_off + n_w * 4])
    out += b"\0" * (end - len(out))
    if records:
        out += TUNE_MAGIC + struct.pack("<q", len(records))
        for r in records:
            if len(r) != TUNE_WORDS:
                raise ValueError("tuning records have %d fields" % TUNE_WORDS)
            out += struct.pack("<%dq" % TUNE_WORDS, *[int(v) for v in r])
    return bytes(out)


def tuning_of(blob: bytes):
    """The tuning records carried by a blob (empty list when it has none)."""
    n_w, _, w_off = struct.unpack_from("<3q", blob, 9 * 8)
    end = (w_off + n_w * 4 + 7) // 8 * 8
    if len(blob) < end + 16 or blob[end:end + 8] != TUNE_MAGIC:
        return []
    (n,) = struct.unpack_from("<q", blob, end + 8)
    return [list(struct.unpack_from("<%dq" % TUNE_WORDS, blob, end + 16 + i * TUNE_WORDS * 8)) for i in range(n)]


def serialize(g: IRGraph, *, enable_fusion: bool, bias_first_fused: bool, kernel_policy: str = "auto",
              fold_epilogues: bool = True) -> bytes:
    live = _live_nodes(g)
    remap: Dict[int, int] = {old: new for new, old in enumerate(live)}
    flags = (FLAG_DYNAMIC if g.dynamic else 0) | (FLAG_FUSION if enable_fusion else 0) \
        | (FLAG_BIAS_FIRST_FUSED if bias_first_fused else 0) | (0 if fold_epilogues else FLAG_NO_FOLD)
    if kernel_policy not in POLICIES:
        raise ValueError("unknown gpu kernel policy '%s' (valid: %s)" % (kernel_policy, sorted(POLICIES)))
    in_shape = g.nodes[g.input_id].shape
    static_batch = in_shape[0] if in_shape and in_shape[0] != -1 else 1

    records = []
    weights = []
    w_floats = 0
    for old in live:
        n = g.nodes[old]
        if len(n.inputs) > 4 or len(n.shape) > 4:
            raise ValueError("node %s: too many inputs or dimensions" % n.name)
        ins = [remap[i] for i in n.inputs] + [-1] * (4 - len(n.inputs))
        dims = list(n.shape) + [0] * (4 - len(n.shape))
        c = n.conv or {}
        off = cnt = 0
        if n.op == "CONST":
            pad = (-w_floats) % 16
            if pad:
                weights.append(np.zeros(pad, np.float32))
                w_floats += pad
            arr = np.ascontiguousarray(n.const, dtype=np.float32).ravel()
            off, cnt = w_floats, arr.size
            weights.append(arr)
            w_floats += arr.size
        records.append([remap[old], OPS[n.op], len(n.inputs)] + ins + [len(n.shape)] + dims
                       + [c.get("sh", 1), c.get("sw", 1), c.get("ph", 0), c.get("pw", 0),
                          c.get("dh", 1), c.get("dw", 1), off, cnt])
    nodes_off = HEADER_WORDS * 8
    w_off = nodes_off + len(records) * NODE_WORDS * 8
    w_off = (w_off + 63) // 64 * 64
    header = struct.pack("<8s11q", MAGIC, VERSION, len(records), remap[g.input_id], remap[g.output_id],
                         g.max_batch_size, flags, POLICIES[kernel_policy], static_batch, w_floats,
                         nodes_off, w_off)
    body = b"".join(struct.pack("<%dq" % NODE_WORDS, *r) for r in records)
    blob = bytearray(header + body)
    blob += b"\0" * (w_off - len(blob))
    for w in weights:
        blob += w.tobytes()
    return bytes(blob)


def blob_sha256(blob: bytes) -> str:
    return hashlib.sha256(blob).hexdigest()
