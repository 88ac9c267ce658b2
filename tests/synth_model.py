"""Host copies of the seeded synthetic models that gb_model_synthesize and
gb_model_fill_kv build on the device (one GPU), for the reference forward().

Weight streams (src/engine/loader.c:506-510 shapes, rows = output features):
  layer l, matrix i (wq, wk, wv, wo, gate, up, down) -> stream l * 7 + i + 1,
  Q4_K except wv and ffn_down (Q6_K); embedding Q4_K stream 1000001; output
  head Q6_K stream 1000002; every RMSNorm weight 1.0.
K / V fill: layer l, K (0) or V (1), KV head h -> ~N(0, 1) stream
  (l * 2 + which) * 256 + h + 5000000, n_pos x head_dim values per head.
"""
import numpy as np

DTYPES = (4, 4, 5, 4, 4, 4, 5)


class Synth:
    pass


def gpu_blocks(gb, torch):
    """A block generator that runs gb_synth_blocks on the device and copies
    the bytes to the host: the same bytes as oracle.synth_blocks (pinned by
    tests/test_gpu_quant.py::test_synth_bytes_match_cpu_generator), made in
    milliseconds instead of seconds for the 128256-row tables."""
    def gen(dtype, rows, cols, seed, stream):
        nblk = rows * (cols // gb.BLOCK_WIDTH[dtype])
        buf = torch.empty(nblk * gb.BLOCK_BYTES[dtype], dtype=torch.uint8, device="cuda")
        gb.synth_blocks(dtype, buf, nblk, seed, stream)
        torch.cuda.synchronize()
        return buf.cpu().numpy()
    return gen


def synth_model(oracle, H, n_heads, n_kv, n_layers, ff, vocab, max_seq, seed, gen=None):
    gen = gen or oracle.synth_blocks
    m = Synth()
    m.H, m.n_heads, m.n_kv, m.hd, m.ff = H, n_heads, n_kv, H // n_heads, ff
    m.vocab, m.n_layers, m.max_seq = vocab, n_layers, max_seq
    kv = n_kv * m.hd
    shapes = [(H, H), (kv, H), (kv, H), (H, H), (ff, H), (ff, H), (H, ff)]
    ones = np.ones(H, np.float32)
    m.layers = []
    for l in range(n_layers):
        L = Synth()
        L.w = [gen(dt, r, c, seed, l * 7 + i + 1) for i, (dt, (r, c)) in enumerate(zip(DTYPES, shapes))]
        L.dtypes = list(DTYPES)
        L.rms_att = ones
        L.rms_ffn = ones
        m.layers.append(L)
    m.emb_dtype, m.lm_dtype = 4, 5
    m.embedding = gen(4, vocab, H, seed, 1000001)
    m.lm_head = gen(5, vocab, H, seed, 1000002)
    m.rms_final = ones
    return m


def fill_kv(oracle, ref, m, n_pos, seed):
    """The reference model's caches filled as gb_model_fill_kv fills the
    device caches."""
    for l in range(m.n_layers):
        for which in (0, 1):
            buf = ref.kv(l, which, m.n_kv * m.max_seq * m.hd).reshape(m.n_kv, m.max_seq, m.hd)
            for h in range(m.n_kv):
                buf[h, :n_pos] = oracle.synth_normal(n_pos * m.hd, seed,
                                                     (l * 2 + which) * 256 + h + 5000000).reshape(n_pos, m.hd)
