"""Parameter layout helper for the tests (GPTModel::parameters() order)."""
import numpy as np


def param_slices(cfg):
    d, f, v = cfg["dim"], cfg["ffn"], cfg["vocab"]
    names = [("embed", (v, d))]
    for l in range(cfg["layers"]):
        names += [(f"l{l}.rms_attn", (d,)), (f"l{l}.wq", (d, d)), (f"l{l}.wk", (d, d)),
                  (f"l{l}.wv", (d, d)), (f"l{l}.wo", (d, d)), (f"l{l}.rms_ffn", (d,)),
                  (f"l{l}.wgate", (f, d)), (f"l{l}.wup", (f, d)), (f"l{l}.wdown", (d, f))]
    names.append(("rms_final", (d,)))
    off = 0
    out = []
    for n, s in names:
        k = int(np.prod(s))
        out.append((n, slice(off, off + k)))
        off += k
    return out
