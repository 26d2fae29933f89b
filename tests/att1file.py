"""Writer for .att1 model files (test helper).

Produces version-1 files in the layout att1_model_load reads (header 80 B,
config 9 x u32, 128-byte tensor descriptors, data section), from the seeded
synthetic weights of the oracle, so that the file-loading path of the
library and of the reference can be run on identical bytes.
"""
import struct

import numpy as np

F32, Q8, Q4 = 1, 2, 3


def write(path, config, tensors):
    """config: dict with vocab_size, n_layers, n_heads, d_model, d_ff,
    max_seq_len; tensors: list of (name, dtype, shape, payload bytes, flags)."""
    header = 80
    cfg = struct.pack("<9I", config["vocab_size"], config["n_layers"], config["n_heads"],
                      config["d_model"], config["d_ff"], config["max_seq_len"],
                      config.get("rope_dim", 0), 1, 0)
    cfg_off = header
    desc_off = cfg_off + len(cfg)
    data_off = desc_off + 128 * len(tensors)
    data_off = (data_off + 63) // 64 * 64
    descs, blobs, off = [], [], 0
    for name, dtype, shape, payload, flags in tensors:
        shp = list(shape) + [0] * (4 - len(shape))
        descs.append(name.encode().ljust(64, b"\0") +
                     struct.pack("<II4QQQII", dtype, len(shape), *shp, off, len(payload), 0, flags))
        pad = (-len(payload)) % 64
        blobs.append(payload + b"\0" * pad)
        off += len(payload) + pad
    data = b"".join(blobs)
    hdr = b"ATT1MODL" + struct.pack("<II8Q", 1, header, cfg_off, len(cfg), desc_off, len(tensors),
                                    data_off, len(data), 0, 0)
    with open(path, "wb") as f:
        f.write(hdr)
        f.write(cfg)
        f.write(b"".join(descs))
        f.write(b"\0" * (data_off - desc_off - 128 * len(tensors)))
        f.write(data)


def synth_model_file(path, orc, vocab, n_layers, n_heads, d_model, d_ff, max_seq, dtype, seed):
    """Synthetic model (norm gains 1, matrices N(0, 0.02)) as a .att1 file.
    dtype 'q4': q4 [out][in] tensors (group 32, flags 32); 'f32': f32
    [in][out] tensors as the reference's f32 models store them (the q8 path
    quantises those at run time)."""
    import oracle as O
    d, f, V = d_model, d_ff, vocab
    ones = np.ones(d, np.float32).tobytes()
    t = [("tok_embeddings.weight", F32, (V, d),
          orc.synth_normal(seed, O.T_EMBED, V * d).tobytes(), 0)]

    def mat(name, tid, rows, cols):
        w = orc.synth_normal(seed, tid, rows * cols).reshape(rows, cols)
        if dtype == "q4":
            p, s = orc.q4_quantize(w)
            return (name, Q4, (rows, cols), p.tobytes() + s.tobytes(), 32)
        return (name, F32, (cols, rows), np.ascontiguousarray(w.T).tobytes(), 0)

    for l in range(n_layers):
        b = l * O.T_PER_LAYER
        p = f"layers.{l}."
        t.append((p + "attention_norm.weight", F32, (d,), ones, 0))
        t.append(mat(p + "attention.wq.weight", b + O.T_WQ, d, d))
        t.append(mat(p + "attention.wk.weight", b + O.T_WK, d, d))
        t.append(mat(p + "attention.wv.weight", b + O.T_WV, d, d))
        t.append(mat(p + "attention.wo.weight", b + O.T_WO, d, d))
        t.append((p + "ffn_norm.weight", F32, (d,), ones, 0))
        t.append(mat(p + "ffn.w_gate.weight", b + O.T_GATE, f, d))
        t.append(mat(p + "ffn.w_up.weight", b + O.T_UP, f, d))
        t.append(mat(p + "ffn.w_down.weight", b + O.T_DOWN, d, f))
    t.append(("output_norm.weight", F32, (d,), ones, 0))
    t.append(mat("output.weight", O.T_OUTPUT, V, d))
    write(path, dict(vocab_size=V, n_layers=n_layers, n_heads=n_heads, d_model=d, d_ff=f,
                     max_seq_len=max_seq), t)
