"""GGUF files: reading, writing, and loading a model onto the GPU.

Reader (GgufModelIndex::parse_file, gguf_loader.rs:142-247): the magic
"GGUF", version (2 or 3), tensor and key-value counts, the typed metadata,
the tensor table (name, dims with the row length first, GGML type, offset
relative to the data section), and the data section at the first multiple of
`general.alignment` (default 32, at least 32) after the table.  Tensor data is
memory-mapped, not read, until a tensor is uploaded.

Writer: the same layout (version 3), used to make synthetic model files for
tests and benchmarks (the reference ships no model files; a real Q4_K_M file
loads the same way).

Loader (ModelConfig::from_gguf and resolve_layers, smollm_chat.rs:67-126,
:214-278; Model::load, :1905-2154): the architecture's hyper-parameters from
the metadata, the tensors by their GGUF names (blk.N.attn_q.weight, ...,
ffn_gate_inp / ffn_gate_exps / ffn_up_exps / ffn_down_exps for MoE layers, a
missing output.weight meaning the LM head is tied to token_embd), every tensor
uploaded to the device and handed to spindle_b200.decoder.Decoder, which
repacks the K-quant matrices to TILED16.
"""
import struct

import numpy as np

GGUF_MAGIC = 0x46554747  # "GGUF" little-endian
DEFAULT_ALIGNMENT = 32

# GGUF metadata value types
T_U8, T_I8, T_U16, T_I16, T_U32, T_I32, T_F32, T_BOOL, T_STRING, T_ARRAY, T_U64, T_I64, T_F64 = range(13)
_SCALAR = {T_U8: "<B", T_I8: "<b", T_U16: "<H", T_I16: "<h", T_U32: "<I", T_I32: "<i", T_F32: "<f", T_BOOL: "<?",
           T_U64: "<Q", T_I64: "<q", T_F64: "<d"}

# GGML types: (weights per block, bytes per block) (quant.rs:1527-1542)
GGML_BLOCK = {0: (1, 4), 1: (1, 2), 2: (32, 18), 3: (32, 20), 6: (32, 22), 7: (32, 24), 8: (32, 34), 12: (256, 144),
              13: (256, 176), 14: (256, 210), 30: (1, 2)}


class GgufError(ValueError):
    pass


def tensor_bytes(dtype, dims):
    """Bytes of a tensor of GGML type `dtype` with dims [row length, rows, ...]."""
    if dtype not in GGML_BLOCK:
        raise GgufError("unsupported GGML type %d" % dtype)
    blk, nb = GGML_BLOCK[dtype]
    if dims[0] % blk:
        raise GgufError("row length %d is not a multiple of the block size %d" % (dims[0], blk))
    n = 1
    for d in dims[1:]:
        n *= int(d)
    return int(dims[0]) // blk * nb * n


class _Reader:
    def __init__(self, buf):
        self.buf, self.pos = buf, 0

    def take(self, n):
        if self.pos + n > len(self.buf):
            raise GgufError("truncated GGUF header")
        b = self.buf[self.pos:self.pos + n]
        self.pos += n
        return bytes(b)

    def scalar(self, t):
        fmt = _SCALAR[t]
        return struct.unpack(fmt, self.take(struct.calcsize(fmt)))[0]

    def string(self):
        n = self.scalar(T_U64)
        if n > (16 << 20):
            raise GgufError("GGUF string length exceeds 16 MiB")
        return self.take(n).decode("utf-8", errors="replace")

    def value(self, t):
        if t in _SCALAR:
            return self.scalar(t)
        if t == T_STRING:
            return self.string()
        if t == T_ARRAY:
            et, n = self.scalar(T_U32), self.scalar(T_U64)
            if et == T_STRING:
                return [self.string() for _ in range(n)]
            if et not in _SCALAR:
                raise GgufError("unknown GGUF array element type %d" % et)
            fmt = _SCALAR[et]
            sz = struct.calcsize(fmt)
            return list(np.frombuffer(self.take(sz * n), dtype=np.dtype(fmt)))
        raise GgufError("unknown GGUF value type %d" % t)


class GgufTensor:
    def __init__(self, name, dims, dtype, rel_offset):
        self.name, self.dims, self.dtype, self.rel_offset = name, list(dims), dtype, rel_offset
        self.offset = None  # absolute, set once the data section is known
        self.nbytes = tensor_bytes(dtype, dims)


class GgufFile:
    """A parsed GGUF file: .version, .alignment, .metadata (key -> value),
    .tensors (name -> GgufTensor, in file order), .data(name) -> uint8 view."""

    def __init__(self, path):
        self.path = path
        self._map = np.memmap(path, dtype=np.uint8, mode="r")
        r = _Reader(self._map)
        if r.scalar(T_U32) != GGUF_MAGIC:
            raise GgufError("not a GGUF file")
        self.version = r.scalar(T_U32)
        if self.version not in (2, 3):
            raise GgufError("unsupported GGUF version %d" % self.version)
        n_tensors, n_kv = r.scalar(T_U64), r.scalar(T_U64)
        self.metadata = {}
        for _ in range(n_kv):
            key = r.string()
            self.metadata[key] = r.value(r.scalar(T_U32))
        a = self.metadata.get("general.alignment", DEFAULT_ALIGNMENT)
        self.alignment = max(int(a), DEFAULT_ALIGNMENT)
        self.tensors = {}
        for _ in range(n_tensors):
            name = r.string()
            nd = r.scalar(T_U32)
            dims = [r.scalar(T_U64) for _ in range(nd)]
            dtype = r.scalar(T_U32)
            self.tensors[name] = GgufTensor(name, dims, dtype, r.scalar(T_U64))
        self.data_offset = -(-r.pos // self.alignment) * self.alignment
        end = 0
        for t in self.tensors.values():
            t.offset = self.data_offset + t.rel_offset
            end = max(end, t.offset + t.nbytes)
        if end > len(self._map):
            # Model::load's check (smollm_chat.rs:1958-1978): a cut-off download
            raise GgufError("the file is incomplete: its tensors need %d bytes, it has %d" % (end, len(self._map)))
        self.architecture = self.metadata.get("general.architecture", "")

    def data(self, name):
        t = self.tensors[name]
        return self._map[t.offset:t.offset + t.nbytes]


def _put_value(out, v, t=None):
    if t is None:
        if isinstance(v, bool):
            t = T_BOOL
        elif isinstance(v, (int, np.integer)):
            t = T_U32 if 0 <= int(v) < 2 ** 32 else T_I64
        elif isinstance(v, (float, np.floating)):
            t = T_F32
        elif isinstance(v, str):
            t = T_STRING
        elif isinstance(v, (list, tuple)):
            t = T_ARRAY
        else:
            raise GgufError("cannot store %r in GGUF metadata" % (v,))
    out.append(struct.pack("<I", t))
    if t in _SCALAR:
        out.append(struct.pack(_SCALAR[t], v))
    elif t == T_STRING:
        b = v.encode("utf-8")
        out.append(struct.pack("<Q", len(b)) + b)
    else:
        et = T_STRING if v and isinstance(v[0], str) else (T_F32 if v and isinstance(v[0], float) else T_I32)
        out.append(struct.pack("<IQ", et, len(v)))
        for x in v:
            if et == T_STRING:
                b = x.encode("utf-8")
                out.append(struct.pack("<Q", len(b)) + b)
            else:
                out.append(struct.pack(_SCALAR[et], x))


def write_gguf(path, metadata, tensors, alignment=DEFAULT_ALIGNMENT):
    """Writes a GGUF v3 file.  metadata: key -> value (bool, int, float, str,
    or a list of those; (value, type) tuples pin a type); tensors: list of
    (name, dims [row length, rows, ...], GGML type, bytes)."""
    meta = dict(metadata)
    if alignment != DEFAULT_ALIGNMENT:
        meta["general.alignment"] = (alignment, T_U32)
    head = [struct.pack("<IIQQ", GGUF_MAGIC, 3, len(tensors), len(meta))]
    for k, v in meta.items():
        kb = k.encode("utf-8")
        head.append(struct.pack("<Q", len(kb)) + kb)
        if isinstance(v, tuple):
            _put_value(head, v[0], v[1])
        else:
            _put_value(head, v)
    off, offs = 0, []
    for name, dims, dtype, data in tensors:
        n = tensor_bytes(dtype, dims)
        if len(data) != n:
            raise GgufError("%s: %d bytes for dims %s of type %d (want %d)" % (name, len(data), dims, dtype, n))
        offs.append(off)
        off = -(-(off + n) // alignment) * alignment
    for (name, dims, dtype, _), o in zip(tensors, offs):
        nb = name.encode("utf-8")
        head.append(struct.pack("<Q", len(nb)) + nb + struct.pack("<I", len(dims)))
        head.append(struct.pack("<%dQ" % len(dims), *[int(d) for d in dims]) + struct.pack("<IQ", dtype, o))
    h = b"".join(head)
    pad = -len(h) % alignment
    with open(path, "wb") as f:
        f.write(h + b"\0" * pad)
        pos = 0
        for (name, dims, dtype, data), o in zip(tensors, offs):
            f.write(b"\0" * (o - pos))
            b = np.ascontiguousarray(data).reshape(-1).view(np.uint8)
            f.write(b.tobytes())
            pos = o + b.nbytes


# ---- model configuration and tensors -----------------------------------------

_NEOX = {"qwen2": True, "qwen2moe": True, "qwen3": True, "qwen3moe": True, "olmoe": True, "llama": False,
         "granite": False, "granitemoe": False}


def model_config(g):
    """ModelConfig::from_gguf (smollm_chat.rs:67-116) as the decoder's cfg dict."""
    arch = g.architecture
    if arch not in _NEOX:
        raise GgufError("unsupported architecture `%s`" % arch)
    get = lambda k, d=None: g.metadata.get("%s.%s" % (arch, k), d)

    def req(k):
        v = get(k)
        if v is None:
            raise GgufError("GGUF metadata missing `%s.%s`" % (arch, k))
        return int(v)

    if get("expert_gating_func") not in (None, 1):
        raise GgufError("only softmax expert gating is supported")
    dim, n_heads = req("embedding_length"), req("attention.head_count")
    n_kv = int(get("attention.head_count_kv", n_heads))
    head_dim = int(get("attention.key_length", dim // n_heads))
    n_expert = int(get("expert_count", 0))
    vocab = g.metadata.get("tokenizer.ggml.tokens")
    emb = g.tensors.get("token_embd.weight")
    cfg = dict(dim=dim, n_heads=n_heads, n_kv_heads=n_kv, head_dim=head_dim, n_layers=req("block_count"),
               vocab=len(vocab) if vocab else int(emb.dims[1]), max_seq=int(get("context_length", 2048)),
               rope_theta=float(get("rope.freq_base", 10000.0)),
               rms_eps=float(get("attention.layer_norm_rms_epsilon", 1e-5)), rope_neox=_NEOX[arch],
               embedding_scale=float(get("embedding_scale", 1.0)), residual_scale=float(get("residual_scale", 1.0)),
               attn_scale=float(get("attention.scale", 0.0)))
    if head_dim % 8 or n_heads % n_kv:
        raise GgufError("unsupported head layout")
    if "blk.0.attn_q_norm.weight" not in g.tensors:
        cfg["qk_norm"] = False
    if n_expert:
        norm = get("expert_weights_norm")
        cfg["moe"] = dict(n_expert=n_expert, n_used=min(int(get("expert_used_count", 0)), n_expert),
                          n_ff=int(get("expert_feed_forward_length", 0)) or int(g.tensors["blk.0.ffn_gate_exps.weight"].dims[1]),
                          norm=bool(norm) if norm is not None else arch not in ("qwen2moe", "olmoe"))
    else:
        cfg["n_ff"] = int(get("feed_forward_length", 0)) or int(g.tensors["blk.0.ffn_gate.weight"].dims[1])
    return cfg


# decoder weight name -> GGUF tensor name (resolve_layers, smollm_chat.rs:214-278)
def gguf_names(cfg):
    m = {"embed": "token_embd.weight", "head": "output.weight", "out_norm": "output_norm.weight"}
    for i in range(cfg["n_layers"]):
        p, b = "l%d." % i, "blk.%d." % i
        m.update({p + "attn_norm": b + "attn_norm.weight", p + "ffn_norm": b + "ffn_norm.weight",
                  p + "q_norm": b + "attn_q_norm.weight", p + "k_norm": b + "attn_k_norm.weight",
                  p + "wq": b + "attn_q.weight", p + "wk": b + "attn_k.weight", p + "wv": b + "attn_v.weight",
                  p + "wo": b + "attn_output.weight"})
        if cfg.get("moe"):
            m.update({p + "router": b + "ffn_gate_inp.weight", p + "gate_exps": b + "ffn_gate_exps.weight",
                      p + "up_exps": b + "ffn_up_exps.weight", p + "down_exps": b + "ffn_down_exps.weight"})
        else:
            m.update({p + "gate": b + "ffn_gate.weight", p + "up": b + "ffn_up.weight", p + "down": b + "ffn_down.weight"})
    return m


def _dims(cfg, name):
    """GGUF dims [row length, rows(, experts)] of a decoder weight."""
    c, dim, hd = cfg, cfg["dim"], cfg["head_dim"]
    q_dim, kv_dim = c["n_heads"] * hd, c["n_kv_heads"] * hd
    if name in ("embed", "head"):
        return [dim, c["vocab"]]
    if name == "out_norm":
        return [dim]
    k = name.split(".", 1)[1]
    moe = c.get("moe") or {}
    return {"attn_norm": [dim], "ffn_norm": [dim], "q_norm": [hd], "k_norm": [hd], "wq": [dim, q_dim],
            "wk": [dim, kv_dim], "wv": [dim, kv_dim], "wo": [q_dim, dim], "router": [dim, moe.get("n_expert", 0)],
            "gate_exps": [dim, moe.get("n_ff", 0), moe.get("n_expert", 0)],
            "up_exps": [dim, moe.get("n_ff", 0), moe.get("n_expert", 0)],
            "down_exps": [moe.get("n_ff", 0), dim, moe.get("n_expert", 0)],
            "gate": [dim, c.get("n_ff", 0)], "up": [dim, c.get("n_ff", 0)], "down": [c.get("n_ff", 0), dim]}[k]


def write_model(path, cfg, weights, dtypes, arch=None, tie_head=False):
    """A model as a GGUF file: cfg (the decoder's dict), weights (name ->
    numpy bytes or float32 array, or a CUDA tensor), dtypes (name -> GGML type of
    each matrix).  tie_head: omit output.weight (the LM head is token_embd)."""
    moe = cfg.get("moe")
    arch = arch or ("qwen3moe" if moe else "qwen3")
    meta = {"general.architecture": arch, "general.name": "spindle-b200 synthetic %s" % arch,
            arch + ".embedding_length": cfg["dim"], arch + ".block_count": cfg["n_layers"],
            arch + ".attention.head_count": cfg["n_heads"], arch + ".attention.head_count_kv": cfg["n_kv_heads"],
            arch + ".attention.key_length": cfg["head_dim"], arch + ".context_length": cfg["max_seq"],
            arch + ".rope.freq_base": float(cfg["rope_theta"]),
            arch + ".attention.layer_norm_rms_epsilon": float(cfg["rms_eps"]),
            "tokenizer.ggml.tokens": ["<t%d>" % i for i in range(cfg["vocab"])]}
    if moe:
        meta.update({arch + ".expert_count": moe["n_expert"], arch + ".expert_used_count": moe["n_used"],
                     arch + ".expert_feed_forward_length": moe["n_ff"],
                     arch + ".expert_weights_norm": bool(moe.get("norm", True))})
    else:
        meta[arch + ".feed_forward_length"] = cfg["n_ff"]
    names = gguf_names(cfg)
    tensors = []
    for k, gname in names.items():
        if k not in weights or (k == "head" and tie_head):
            continue
        v = weights[k]
        if hasattr(v, "cpu"):
            v = v.cpu().numpy()
        v = np.ascontiguousarray(v)
        dt = dtypes.get(k, 0) if v.dtype == np.uint8 else 0
        tensors.append((gname, _dims(cfg, k), dt, v.reshape(-1).view(np.uint8)))
    write_gguf(path, meta, tensors)


def load_weights(g, cfg, device):
    """Every tensor of the decoder uploaded to `device`: (weights, dtypes),
    the LM head tied to the embedding when output.weight is absent."""
    import torch
    names = gguf_names(cfg)
    weights, dtypes = {}, {}
    for k, gname in names.items():
        t = g.tensors.get(gname)
        if t is None:
            if k == "head":
                t = g.tensors["token_embd.weight"]  # tied (smollm_chat.rs:1921)
            elif k.endswith("q_norm") or k.endswith("k_norm"):
                continue
            else:
                raise GgufError("missing tensor %s" % gname)
        data = np.asarray(g.data(t.name))
        if t.dtype == 0 and len(t.dims) == 1:
            weights[k] = torch.from_numpy(data.view(np.float32).copy()).to(device)
        elif t.dtype == 0 and k.endswith("router"):
            weights[k] = torch.from_numpy(data.view(np.float32).reshape(t.dims[1], t.dims[0]).copy()).to(device)
        else:
            weights[k] = torch.from_numpy(data.copy()).to(device)
        dtypes[k] = t.dtype
    return weights, dtypes


def load_decoder(path, device, max_seq=None, ep=None):
    """Model::load (smollm_chat.rs:1905-2154) onto the GPU: the config from the
    metadata, every tensor uploaded, then a spindle_b200.decoder.Decoder."""
    from .decoder import Decoder
    g = GgufFile(path)
    cfg = model_config(g)
    if max_seq:
        cfg["max_seq"] = max_seq
    weights, dtypes = load_weights(g, cfg, device)
    return Decoder(cfg, weights, dtypes, device, ep=ep), cfg
