"""GGUF v3 files for the loader tests: header, metadata, tensor infos and
the aligned data section (the layout qma_load reads, gguf.c:104-316).
Test infrastructure: writes files, computes nothing."""
import struct

GV = {"u8": 0, "i8": 1, "u16": 2, "i16": 3, "u32": 4, "i32": 5, "f32": 6, "bool": 7, "str": 8, "arr": 9,
      "u64": 10, "i64": 11, "f64": 12}
_FMT = {"u8": "<B", "i8": "<b", "u16": "<H", "i16": "<h", "u32": "<I", "i32": "<i", "f32": "<f", "bool": "<?",
        "u64": "<Q", "i64": "<q", "f64": "<d"}
# bytes per block and elements per block of the weight types
BLOCK = {0: (4, 1), 8: (34, 32), 12: (144, 256), 14: (210, 256), 2: (18, 32)}


def _str(s) -> bytes:
    s = s.encode() if isinstance(s, str) else s
    return struct.pack("<Q", len(s)) + s


def _val(t, v) -> bytes:
    if t == "str":
        return _str(v)
    if t == "arr":
        at, items = v
        return struct.pack("<IQ", GV[at], len(items)) + b"".join(_val(at, x) for x in items)
    return struct.pack(_FMT[t], v)


def tensor_bytes(typ, ne):
    bs, blk = BLOCK[typ]
    n = 1
    for d in ne[1:]:
        n *= d
    return ne[0] // blk * bs * n


def qwen35moe_kv(prefix="qwen35moe.", block_count=40, alignment=None, extra=()):
    """The metadata qma_load reads: hyper-parameters, a small tokenizer
    (tokens and merges that resolve), plus `extra` entries."""
    toks = ["a", "b", "c", "ab", "bc", "abc", "<|im_start|>", "<|im_end|>"] + [f"t{i}" for i in range(56)]
    kv = [("general.architecture", "str", "qwen35moe"),
          (prefix + "block_count", "u32", block_count),
          (prefix + "embedding_length", "u32", 2048),
          (prefix + "attention.head_count", "u32", 16),
          (prefix + "attention.head_count_kv", "u32", 2),
          (prefix + "rope.dimension_count", "u32", 64),
          (prefix + "rope.dimension_sections", "arr", ("i32", [11, 11, 10, 0])),
          (prefix + "rope.freq_base", "f32", 1e7),
          ("tokenizer.ggml.tokens", "arr", ("str", toks)),
          ("tokenizer.ggml.token_type", "arr", ("i32", [1] * 6 + [3, 3] + [1] * 56)),
          ("tokenizer.ggml.merges", "arr", ("str", ["a b", "b c", "ab c"]))]
    if alignment is not None:
        kv.append(("general.alignment", "u32", alignment))
    return kv + list(extra)


def write(path, kv, tensors, data=None, data_size=None, alignment=32, version=3, truncate_by=0):
    """tensors: (name, type, ne, offset in the data section).  The data
    section is `data` (bytes-like) or, with data=None, a sparse run of
    zeros of data_size bytes.  Returns the data section's file offset."""
    hdr = b"GGUF" + struct.pack("<IQQ", version, len(tensors), len(kv))
    hdr += b"".join(_str(k) + struct.pack("<I", GV[t]) + _val(t, v) for k, t, v in kv)
    for name, typ, ne, off in tensors:
        hdr += _str(name) + struct.pack("<I", len(ne)) + b"".join(struct.pack("<Q", d) for d in ne)
        hdr += struct.pack("<IQ", typ, off)
    start = len(hdr) + (-len(hdr)) % alignment
    with open(path, "wb") as f:
        f.write(hdr + b"\0" * (start - len(hdr)))
        if data is not None:
            f.write(data)
            end = start + len(data)
        else:
            end = start + data_size
        f.truncate(end - truncate_by)
    return start


def small_layout(arr, n, alignment=32, override=None):
    """Every tensor of a synthetic qwen35moe layout with one row (names and
    types kept; qma_load checks presence, not shapes), packed at
    `alignment`.  override: {name: (type, ne)}."""
    out, off = [], 0
    for i in range(n):
        name = arr[i].name.decode()
        typ, ne = int(arr[i].type), [int(arr[i].ne[0])]
        if int(arr[i].ne[1]) > 1 or int(arr[i].ne[2]) > 1:
            ne.append(1)
        if int(arr[i].ne[2]) > 1:
            ne.append(2)
        if override and name in override:
            typ, ne = override[name]
        out.append((name, typ, tuple(ne), off))
        off += tensor_bytes(typ, ne)
        off += (-off) % alignment
    return out, off
