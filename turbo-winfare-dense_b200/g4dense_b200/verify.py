"""Integrity check of a `.g4dense` or `.g4mtp` container: what tools/verify_weights.py and
tools/verify_assistant_weights.py of the reference check, in one tool that recognises the file
by its magic word.

* the magic word and format version;
* each block (the embedding, LM head, per-layer-input and layer blocks of a model; the embedding, pre-/post-
  projection, norm and layer sections of an assistant) starts on a 4096-byte boundary, is not
  empty and ends inside the file (for a model, as tools/verify_weights.py:52-62 checks its layers);
* the SHA-256 of everything after the 4096-byte header equals the header's payload digest
  (tools/verify_weights.py:64-79, tools/verify_assistant_weights.py:75-87). The file is hashed in
  64 MiB reads, so a 17 GB container is never held in memory.

The engine's loader does not hash the payload (that would add a pass over the whole file to
every start); run this after copying or downloading a container.

    python -m g4dense_b200.verify model.g4dense [assistant.g4mtp ...]
"""
from __future__ import annotations

import argparse
import hashlib
import struct
import sys
from pathlib import Path

from .container import ALIGNMENT, HEADER_FMT, HEADER_SIZE, MAGIC, MTP_HEADER_FMT, MTP_MAGIC, MTP_MAX_LAYERS, \
    MTP_VERSION, VERSION

_CHUNK = 64 << 20


class ContainerError(ValueError):
    pass


def _blocks_model(raw: bytes) -> tuple:
    """(kind, fields, [(name, offset, size)], declared digest) of a .g4dense header."""
    h = struct.unpack(HEADER_FMT, raw)
    layers = h[3]
    if not 1 <= layers <= 60:
        raise ContainerError(f"{layers} layers; the header's tables hold 1..60")
    offsets, sizes = h[23:83], h[83:143]
    blocks = [("embedding block", h[19], h[20]), ("LM head block", h[21], h[22])]
    if h[146]:  # per-layer inputs (E2B/E4B): their block sits between the head and the layers
        blocks.append(("per-layer-input block", h[150], h[151]))
    blocks += [(f"layer {l}", offsets[l], sizes[l]) for l in range(layers)]
    fields = {"version": h[1], "layers": layers, "d_model": h[4], "d_ff": h[5], "q_heads": h[6], "kv_heads": h[7],
              "head_dim": h[8], "vocab_size": h[9], "sliding_window": h[10], "global_layer_mask": h[14],
              "tied_embeddings": h[13]}
    return "g4dense", fields, blocks, h[143], VERSION


def _blocks_assistant(raw: bytes) -> tuple:
    """The same for a .g4mtp header."""
    h = struct.unpack(MTP_HEADER_FMT, raw)
    layers = h[3]
    if not 1 <= layers <= MTP_MAX_LAYERS:
        raise ContainerError(f"{layers} layers; the header's tables hold 1..{MTP_MAX_LAYERS}")
    blocks = [(name, h[17 + 2 * i], h[18 + 2 * i]) for i, name in
              enumerate(("embedding section", "pre-projection section", "post-projection section", "norm section"))]
    blocks += [(f"layer {l}", h[25 + l], h[33 + l]) for l in range(layers)]
    fields = {"version": h[1], "layers": layers, "backbone": h[4], "hidden": h[5], "intermediate": h[6],
              "vocab_size": h[7], "q_heads": h[8], "kv_heads": h[9], "head_dim": h[10], "global_layer_mask": h[14]}
    return "g4mtp", fields, blocks, h[41], MTP_VERSION


def verify_container(path) -> dict:
    """Checks the container at `path`; returns its kind, header fields and payload digest, or
    raises ContainerError naming the first problem found."""
    p = Path(path)
    if not p.is_file():
        raise ContainerError(f"{p}: no such file")
    size = p.stat().st_size
    with open(p, "rb") as f:
        raw = f.read(HEADER_SIZE)
        if len(raw) != HEADER_SIZE:
            raise ContainerError(f"{p}: {len(raw)} bytes, shorter than the {HEADER_SIZE}-byte header")
        (magic,) = struct.unpack_from("<I", raw)
        if magic == MAGIC:
            kind, fields, blocks, declared, version = _blocks_model(raw)
        elif magic == MTP_MAGIC:
            kind, fields, blocks, declared, version = _blocks_assistant(raw)
        else:
            raise ContainerError(f"{p}: magic word 0x{magic:08X} is neither 'G4DN' (0x{MAGIC:08X}) nor 'G4MT' "
                                 f"(0x{MTP_MAGIC:08X})")
        if fields["version"] != version:
            raise ContainerError(f"{p}: {kind} format version {fields['version']}; expected {version}")
        for name, off, n in blocks:
            if off % ALIGNMENT:
                raise ContainerError(f"{p}: {name} starts at byte {off}, not on a {ALIGNMENT}-byte boundary")
            if n == 0:
                raise ContainerError(f"{p}: {name} is empty")
            if off < HEADER_SIZE or off + n > size:
                raise ContainerError(f"{p}: {name} spans bytes {off}..{off + n}, outside the {size}-byte file")
        sha = hashlib.sha256()
        while chunk := f.read(_CHUNK):
            sha.update(chunk)
    if sha.digest() != declared:
        raise ContainerError(f"{p}: payload SHA-256 {sha.hexdigest()} does not match the header's {declared.hex()}")
    return {"kind": kind, "size": size, "sha256": sha.hexdigest(), **fields}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description="Verify .g4dense / .g4mtp containers (header, blocks, payload SHA-256)")
    ap.add_argument("files", nargs="+", help="container files")
    a = ap.parse_args(argv)
    rc = 0
    for path in a.files:
        try:
            info = verify_container(path)
        except (ContainerError, OSError, struct.error) as e:
            print(f"FAILED {e}", file=sys.stderr)
            rc = 1
            continue
        print(f"OK {path}: {info['kind']} v{info['version']}, {info['layers']} layers, {info['size']:,} bytes, "
              f"payload sha256 {info['sha256']}")
    return rc


if __name__ == "__main__":
    sys.exit(main())
