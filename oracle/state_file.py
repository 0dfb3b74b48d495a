"""Test-infrastructure restatement of optimizer_states.bin version 2
(galore/src/state_file.rs:1-580): header, descriptor table and per-layer
sections, for checking the library's writer and reader byte by byte.  Only
tests import this module; the library has its own C++ implementation.
"""
from __future__ import annotations

import struct

import numpy as np

MAGIC = 0x47414C52            # state_file.rs:22
VERSION = 2                   # :24
HEADER_SIZE = 64              # :26
LAYER_DESC_SIZE = 20          # :28


def layer_state_size(m, n, r):
    """state_file.rs:164-171."""
    return 2 * m * r + 2 * n * r + 2 * r * r + 8


def layer_layout(m, n, r):
    """state_file.rs:193-212: offsets of P, Q, momentum, variance, scale_m, scale_v."""
    q = 2 * m * r
    mo = q + 2 * n * r
    v = mo + r * r
    sm = v + r * r
    return {"p": 0, "q": q, "m": mo, "v": v, "scale_m": sm, "scale_v": sm + 4,
            "size": layer_state_size(m, n, r)}


def build_descriptors(dims, ranks):
    """state_file.rs:217-236: (m, n, rank, byte_offset) per layer."""
    off = HEADER_SIZE + len(dims) * LAYER_DESC_SIZE
    out = []
    for (m, n), r in zip(dims, ranks):
        out.append((m, n, r, off))
        off += layer_state_size(m, n, r)
    return out


def parse_header(buf: bytes):
    """OptimizerStateHeader::from_bytes (state_file.rs:83-131) for version >= 2."""
    magic, version, num_layers, rank, precision, header_size, total = struct.unpack_from("<6IQ", buf, 0)
    beta1, beta2, eps = struct.unpack_from("<3f", buf, 32)
    (step,) = struct.unpack_from("<Q", buf, 44)
    return dict(magic=magic, version=version, num_layers=num_layers, rank=rank, precision=precision,
                header_size=header_size, total_size=total, beta1=beta1, beta2=beta2, eps=eps, step_count=step,
                reserved=bytes(buf[52:64]))


def parse(buf: bytes):
    """Header and layers of a version-2 file (P and Q as their raw f16 bits)."""
    header = parse_header(buf)
    layers = []
    for i in range(header["num_layers"]):
        m, n, r, off = struct.unpack_from("<3IQ", buf, HEADER_SIZE + i * LAYER_DESC_SIZE)
        lay = layer_layout(m, n, r)
        b = off
        layers.append(dict(
            m=m, n=n, rank=r, offset=off,
            p_bits=np.frombuffer(buf, np.uint16, m * r, b + lay["p"]).reshape(m, r),
            q_bits=np.frombuffer(buf, np.uint16, n * r, b + lay["q"]).reshape(n, r),
            m8=np.frombuffer(buf, np.int8, r * r, b + lay["m"]),
            v8=np.frombuffer(buf, np.int8, r * r, b + lay["v"]),
            scale_m=struct.unpack_from("<f", buf, b + lay["scale_m"])[0],
            scale_v=struct.unpack_from("<f", buf, b + lay["scale_v"])[0]))
    return header, layers
