#!/usr/bin/env python3
"""Benchmark: batch-1 greedy decode of the Llama-3.1-8B architecture with a
Q4_K_M-style weight mix, plus the per-kernel HBM rooflines
of configs 0-2 (Q4_K / Q6_K matvec, decode attention).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One process per GPU; for N > 1 launch with torch.distributed.run (RANK,
WORLD_SIZE, LOCAL_RANK from the environment).  Rank 0 prints one JSON line.

Workload (synthetic, seeded; no dataset is involved): random-init weights of
the Llama-3.1-8B shape (32 layers, hidden 4096, 32 q / 8 kv heads, FFN 14336,
vocab 128256) as Q4_K with Q6_K for attn_v, ffn_down and the output head;
the KV context is pre-filled to 4096 positions with seeded ~N(0,1) values,
then K greedy decode steps run from position 4096 + W.  A step is one token
through all 32 layers, the final norm, the output head and the argmax.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

LLAMA8B = dict(hidden_dim=4096, n_heads=32, n_kv_heads=8, n_layers=32, ff_dim=14336, vocab_size=128256)
CTX = 4096
SEED = 1234
METRIC = "decode tokens/s (Llama-3.1-8B arch, Q4_K_M, ctx 4096, batch 1)"
PREFILL_T = 4096


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def bf16_peak():
    """Dense fp16 / bf16 tensor peak: the measured bf16 dense sustained rate."""
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        return float(json.load(open(p))["bf16_tflops_sustained"])
    return 1400.0


def tf32_peak():
    """Dense tf32 tensor peak: half the measured bf16 dense sustained rate."""
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        return float(json.load(open(p))["bf16_tflops_sustained"]) / 2
    return 1400.0 / 2


def ncu_traffic(summary: str = "q4k_gateup_grouped_2x14336x4096.md"):
    """Per-launch DRAM bytes of a dominant kernel from its committed ncu
    summary under profiles/ (the decode step's gate + up launch by default),
    or None."""
    p = os.path.join(ROOT, "profiles", summary)
    if not os.path.exists(p):
        return None
    for line in open(p):
        if line.startswith("traffic_bytes_per_launch:"):
            try:
                return float(line.split(":", 1)[1].strip().split()[0])
            except ValueError:
                return None
    return None


class Clocks:
    """nvidia-smi samples of SM clock and throttle reasons during a region."""
    Q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.p = None

    def __enter__(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--id={self.device}", f"--query-gpu={self.Q}",
                                       "--format=csv,noheader,nounits", "-lms", "100"],
                                      stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.p = None
        time.sleep(0.3)
        return self

    def __exit__(self, *a):
        self.rows = []
        if self.p is None:
            return
        time.sleep(0.15)
        self.p.terminate()
        out, _ = self.p.communicate(timeout=10)
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) == 7:
                self.rows.append(f)

    def summary(self):
        if not getattr(self, "rows", None):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[0]) for r in self.rows if r[0].replace(".", "").isdigit()]
        mx = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows for i in range(4) if r[3 + i].lower().startswith("active")})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.rows)}


# ---------------------------------------------------------------- our arm
def kernel_benchmarks(gb, torch, dm, peak):
    """Isolated kernel timings with CUDA events on the launching stream.
    Every timed launch reads a buffer that is not in L2 (copies rotate over
    more than 4x the 126 MB L2)."""
    st = torch.cuda.Stream()
    sp = st.cuda_stream
    res = {}

    def timed(launch, n_iter, warm=3, reps=3):
        """Seconds per launch: n_iter launches captured in one CUDA graph on
        the launching stream (as the decode step issues them, without host
        overhead), replayed reps times between CUDA events on that stream.
        Matvec launches carry programmatic dependent launch, so each one
        starts fetching weights during its predecessor's tail, as in the
        decode step (GB_DISABLE_PDL=1 in the environment times them
        unchained)."""
        for i in range(warm):
            launch(i)
        st.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=st, capture_error_mode="relaxed"):
            for i in range(n_iter):
                launch(i)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(st):   # replay() launches on the current stream
            g.replay()
            st.synchronize()
            e0.record(st)
            for _ in range(reps):
                g.replay()
            e1.record(st)
        e1.synchronize()
        del g
        return e0.elapsed_time(e1) / (n_iter * reps) * 1e-3

    def matvec_case(tag, dt, rows, cols, copies, n_iter, alg_cols=None):
        # alg_cols: the matrix's real columns when its rows are laid out padded
        # to `cols` (the algorithmic bytes count the real ones)
        wbytes = gb.matrix_bytes(dt, rows, cols)
        bufs = [torch.empty(wbytes + 16, dtype=torch.uint8, device="cuda") for _ in range(copies)]
        nblk = wbytes // gb.BLOCK_BYTES[dt]
        for j, b in enumerate(bufs):
            gb.synth_blocks(dt, b, nblk, SEED, 77 + j, stream=sp)
        x = torch.empty(cols, dtype=torch.float32, device="cuda")
        gb.synth_normal(x, cols, SEED, 5, stream=sp)
        y = torch.empty(rows, dtype=torch.float32, device="cuda")
        st.synchronize()
        t = timed(lambda i: gb.matvec(dt, bufs[i % copies], rows, cols, x, y, stream=sp), n_iter)
        ac = alg_cols or cols
        alg = gb.matrix_bytes(dt, rows, ac) + 4 * ac + 4 * rows
        gbs = alg / t / 1e9
        res[tag] = {"us": round(t * 1e6, 2), "alg_bytes": alg, "GB/s": round(gbs, 1), "frac": round(gbs / peak, 3)}
        del bufs
        torch.cuda.empty_cache()
        return gbs, alg, t

    def gateup_case(tag, rows, cols, copies, n_iter):
        """gate and up as the decode step launches them: one grouped launch
        over two Q4_K matrices that share x."""
        wbytes = gb.matrix_bytes(4, rows, cols)
        bufs = [[torch.empty(wbytes + 16, dtype=torch.uint8, device="cuda") for _ in range(2)] for _ in range(copies)]
        for j, pair in enumerate(bufs):
            for i, b in enumerate(pair):
                gb.synth_blocks(4, b, wbytes // gb.BLOCK_BYTES[4], SEED, 300 + 2 * j + i, stream=sp)
        x = torch.empty(cols, dtype=torch.float32, device="cuda")
        gb.synth_normal(x, cols, SEED, 5, stream=sp)
        ys = [torch.empty(rows, dtype=torch.float32, device="cuda") for _ in range(2)]
        st.synchronize()
        t = timed(lambda i: gb.matvec_group([4, 4], bufs[i % copies], [rows, rows], cols, x, ys, stream=sp), n_iter)
        alg = 2 * wbytes + 4 * cols + 2 * 4 * rows
        gbs = alg / t / 1e9
        res[tag] = {"us": round(t * 1e6, 2), "alg_bytes": alg, "GB/s": round(gbs, 1), "frac": round(gbs / peak, 3)}
        del bufs
        torch.cuda.empty_cache()
        return gbs, alg, t

    main = gateup_case("q4k_gateup_grouped_2x14336x4096", 14336, 4096, 6, 100)
    matvec_case("q4k_matvec_14336x4096", 4, 14336, 4096, 12, 200)
    matvec_case("q4k_matvec_4096x4096 (config 0)", 4, 4096, 4096, 40, 400)
    matvec_case("q6k_matvec_4096x14336 (config 1)", 5, 4096, 14336, 10, 200)
    matvec_case("q6k_matvec_128256x4096 (config 1, output head)", 5, 128256, 4096, 2, 40)
    matvec_case("q8_0_matvec_14336x4096", 2, 14336, 4096, 8, 200)
    matvec_case("q6k_matvec_2048x5632 (config 3 ffn_down, rows padded to 24 blocks as the model lays them out)", 5,
                2048, 6144, 24, 400, alg_cols=5632)

    # config 2: RoPE + append + GQA attention over 8193 positions (fp32 KV)
    nh, nkv, hd, ms, pos = 32, 8, 128, 8448, 8192
    copies = 5
    kv_elems = nkv * ms * hd
    kcs = [torch.empty(kv_elems, dtype=torch.float32, device="cuda") for _ in range(copies)]
    vcs = [torch.empty(kv_elems, dtype=torch.float32, device="cuda") for _ in range(copies)]
    for j in range(copies):
        gb.synth_normal(kcs[j], kv_elems, SEED, 900 + j, stream=sp)
        gb.synth_normal(vcs[j], kv_elems, SEED, 950 + j, stream=sp)
    q = torch.empty(nh * hd, dtype=torch.float32, device="cuda")
    k = torch.empty(nkv * hd, dtype=torch.float32, device="cuda")
    v = torch.empty(nkv * hd, dtype=torch.float32, device="cuda")
    for t_, n_, s_ in ((q, nh * hd, 1), (k, nkv * hd, 2), (v, nkv * hd, 3)):
        gb.synth_normal(t_, n_, SEED, s_, stream=sp)
    cs = torch.empty(ms * hd, dtype=torch.float32, device="cuda")
    gb.rope_table(cs, ms, hd, stream=sp)
    ws = torch.zeros(gb.attn_workspace_bytes(nh, nkv, hd, ms), dtype=torch.uint8, device="cuda")
    d_pos = torch.tensor([pos], dtype=torch.int32, device="cuda")
    out = torch.empty(nh * hd, dtype=torch.float32, device="cuda")
    st.synchronize()
    t = timed(lambda i: gb.attention_decode(q, k, v, kcs[i % copies], vcs[i % copies], cs, d_pos, nh, nkv, hd, ms,
                                            out, ws, stream=sp), 200)
    alg = 2 * nkv * (pos + 1) * hd * 4 + 2 * nkv * hd * 4 + 2 * nh * hd * 4
    gbs = alg / t / 1e9
    res["attention_decode_8193 (config 2)"] = {"us": round(t * 1e6, 2), "alg_bytes": alg, "GB/s": round(gbs, 1),
                                               "frac": round(gbs / peak, 3)}
    del kcs, vcs
    torch.cuda.empty_cache()
    return res, main


TINYLLAMA = dict(hidden_dim=2048, n_heads=32, n_kv_heads=4, n_layers=22, ff_dim=5632, vocab_size=32000)


def tinyllama_decode(gb, torch, prompt_len=128, steps=256):
    """TinyLlama-1.1B architecture, random-init Q4_K_M-style
    weights, a 128-token prompt fed through the decode path, then 256 greedy
    steps (device-timed, CUDA events on the launching stream)."""
    import numpy as np
    c = TINYLLAMA
    dm = gb.DecodeModel(c["hidden_dim"], c["n_heads"], c["n_kv_heads"], c["n_layers"], c["ff_dim"],
                        c["vocab_size"], prompt_len + steps + 8)
    try:
        dm.synthesize(SEED)
        prompt = np.random.RandomState(SEED).randint(0, c["vocab_size"], prompt_len)
        t0 = time.perf_counter()
        nxt = 0
        for pos, tok in enumerate(prompt):
            nxt = dm.decode_host(int(tok), pos)
        t_prompt = time.perf_counter() - t0
        st = torch.cuda.Stream()
        d_tok = torch.tensor([nxt], dtype=torch.int32, device="cuda")
        d_pos = torch.tensor([prompt_len], dtype=torch.int32, device="cuda")
        toks = torch.zeros(steps + 1, dtype=torch.int32, device="cuda")
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        dm.generate(d_tok, d_pos, 3, toks, stream=st.cuda_stream)   # warm-up (graph capture)
        st.synchronize()
        d_tok.fill_(nxt)
        d_pos.fill_(prompt_len)
        st.synchronize()
        e0.record(st)
        dm.generate(d_tok, d_pos, steps, toks, stream=st.cuda_stream)
        e1.record(st)
        e1.synchronize()
        if dm.error() != 0:
            raise RuntimeError(f"decode error {dm.error()}")
        ms = e0.elapsed_time(e1)
        return {"workload": "tinyllama-1.1b-q4km (BASELINE config 3): 128-token prompt, 256 greedy steps",
                "tokens_per_s": round(steps / (ms / 1e3), 1), "ms_per_token": round(ms / steps, 4),
                "prompt_tokens_per_s_host_calls": round(prompt_len / t_prompt, 1),
                "launches_per_step": dm.launches_per_step()}
    finally:
        dm.close()


def one_gpu_tokens(gb, torch, max_seq, W, K):
    """Greedy tokens of the timed steps from a one-GPU model of the same
    seeded weights and KV fill (the tensor-parallel run must reproduce them)."""
    c = LLAMA8B
    dm = gb.DecodeModel(c["hidden_dim"], c["n_heads"], c["n_kv_heads"], c["n_layers"], c["ff_dim"],
                        c["vocab_size"], max_seq)
    try:
        dm.synthesize(SEED)
        dm.fill_kv(CTX, SEED)
        st = torch.cuda.Stream()
        d_tok = torch.tensor([1], dtype=torch.int32, device="cuda")
        d_pos = torch.tensor([CTX], dtype=torch.int32, device="cuda")
        toks = torch.zeros(max(W, K) + 1, dtype=torch.int32, device="cuda")
        dm.generate(d_tok, d_pos, W, toks, stream=st.cuda_stream)
        dm.generate(d_tok, d_pos, K, toks, stream=st.cuda_stream)
        st.synchronize()
        return toks[:K].cpu().tolist()
    finally:
        dm.close()


def _ref_llama_sample(O, n_layers_sample: int, max_seq: int):
    """The reference harness model (oracle/_ref) at the Llama-8B width with
    n_layers_sample seeded layers and the full output head."""
    import numpy as np

    class M:
        pass
    m = M()
    c = LLAMA8B
    m.H, m.n_heads, m.n_kv, m.hd, m.ff = c["hidden_dim"], c["n_heads"], c["n_kv_heads"], 128, c["ff_dim"]
    m.vocab, m.n_layers, m.max_seq = c["vocab_size"], n_layers_sample, max_seq
    m.layers = []
    kv = m.n_kv * m.hd
    shapes = [(m.H, m.H), (kv, m.H), (kv, m.H), (m.H, m.H), (m.ff, m.H), (m.ff, m.H), (m.H, m.ff)]
    dts = [4, 4, 5, 4, 4, 4, 5]
    for li in range(n_layers_sample):
        L = M()
        L.w = [O.synth_blocks(dt, r, cc, SEED, li * 7 + i + 1) for i, (dt, (r, cc)) in enumerate(zip(dts, shapes))]
        L.dtypes = dts
        L.rms_att = np.ones(m.H, np.float32)
        L.rms_ffn = np.ones(m.H, np.float32)
        m.layers.append(L)
    m.emb_dtype, m.lm_dtype = 4, 5
    m.embedding = O.synth_blocks(4, m.vocab, m.H, SEED, 1000001)
    m.lm_head = O.synth_blocks(5, m.vocab, m.H, SEED, 1000002)
    m.rms_final = np.ones(m.H, np.float32)
    return m, O.RefModel(m)


def cpu_reference_token_time(threads: int, n_layers_sample: int = 1, reps: int = 2):
    """Seconds per Llama-8B decode token on the host cores through the
    reference's own forward() (oracle/_ref, compiled unchanged), measured on a
    bounded sample: forward() of a model with n_layers_sample layers plus the
    full output head, and the output-head matvec alone; the token time is
    head + 32 * (sample - head) / n_layers_sample."""
    from oracle import oracle as O
    if not O.ref_available():
        return None
    R = O.ref()
    R.ref_set_threads(threads)
    m, ref = _ref_llama_sample(O, n_layers_sample, CTX + 8)
    for li in range(n_layers_sample):
        for which in (0, 1):
            buf = ref.kv(li, which, m.n_kv * m.max_seq * m.hd).reshape(m.n_kv, m.max_seq, m.hd)
            buf[:, :CTX] = O.synth_normal(m.n_kv * CTX * m.hd, SEED, 77 + which).reshape(m.n_kv, CTX, m.hd)
    x = O.synth_normal(m.H, SEED, 3)
    t_fw, t_head = [], []
    for r in range(reps):
        t0 = time.perf_counter()
        ref.forward(1, CTX + r)
        t_fw.append(time.perf_counter() - t0)
        t0 = time.perf_counter()
        O.ref_matvec(5, m.lm_head, m.vocab, m.H, x)
        t_head.append(time.perf_counter() - t0)
    ref.close()
    R.ref_set_threads(1)
    fw, head = min(t_fw), min(t_head)
    return head + LLAMA8B["n_layers"] * max(fw - head, 0.0) / n_layers_sample


def cpu_reference_prefill_rate(threads: int, T: int = 32):
    """Prompt tokens/s of the reference's CPU prefill (forward() with
    n_tokens = T, oracle/_ref compiled unchanged) at the Llama-8B shape, on a
    bounded sample: one layer plus the output head over a T-token prompt, and
    the head alone; rate = T / (32 x (sample - head)).  The reference's
    linear_dispatch runs its matvec once per prompt row (engine.c:119-153), so
    the per-row cost hardly depends on T."""
    import numpy as np
    from oracle import oracle as O
    if not O.ref_available():
        return None
    R = O.ref()
    R.ref_set_threads(threads)
    m, ref = _ref_llama_sample(O, 1, T + 8)
    prompt = np.random.RandomState(SEED).randint(0, m.vocab, T).astype(np.int32)
    x = O.synth_normal(m.H, SEED, 3)
    t0 = time.perf_counter()
    ref.forward_tokens(prompt, 0)
    t_fw = time.perf_counter() - t0
    t0 = time.perf_counter()
    O.ref_matvec(5, m.lm_head, m.vocab, m.H, x)
    t_head = time.perf_counter() - t0
    ref.close()
    R.ref_set_threads(1)
    layer = max(t_fw - t_head, 1e-9)
    return T / (LLAMA8B["n_layers"] * layer)


def prefill_bench(gb, torch, peak_tf32, T=PREFILL_T, reps=2):
    """Prompt tokens/s of gb_model_prefill on the Llama-3.1-8B shape (32 layers,
    seeded Q4_K_M-style weights): one T-token prompt per step, device-timed
    with CUDA events on the launching stream after one warm-up prefill; e2e
    through gb_model_prefill_host (prompt H2D, next token D2H, synchronous).
    The dominant kernel, the Q4_K GEMM 14336 x 4096 x T (gate or up), is timed
    alone on an X split beforehand (fp16 operands; the split is its own
    launch) for the roofline: tensor rate = 3 products x 2 N K T / time,
    against the fp16 (or, with GB_GEMM_KIND=tf32, the tf32) dense peak."""
    import numpy as np
    c = LLAMA8B
    dm = gb.DecodeModel(c["hidden_dim"], c["n_heads"], c["n_kv_heads"], c["n_layers"], c["ff_dim"],
                        c["vocab_size"], T + 8)
    try:
        dm.synthesize(SEED)
        prompt = np.random.RandomState(SEED).randint(0, c["vocab_size"], T).astype(np.int32)
        st = torch.cuda.Stream()
        d_tok = torch.from_numpy(prompt).to("cuda")
        lg = torch.empty(c["vocab_size"], device="cuda")
        nx = torch.empty(1, dtype=torch.int32, device="cuda")
        torch.cuda.synchronize()
        dm.prefill(d_tok, T, 0, lg, nx, stream=st.cuda_stream)   # warm-up (buffers, smem attributes)
        st.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        for _ in range(reps):
            dm.prefill(d_tok, T, 0, lg, nx, stream=st.cuda_stream)
        e1.record(st)
        e1.synchronize()
        ms = e0.elapsed_time(e1) / reps
        if dm.error() != 0:
            raise RuntimeError(f"prefill error {dm.error()}")
        t0 = time.perf_counter()
        nxt = dm.prefill_host(prompt, 0)
        e2e_s = time.perf_counter() - t0
        # dominant kernel alone
        N, K = c["ff_dim"], c["hidden_dim"]
        nb = gb.matrix_bytes(4, N, K)
        W = torch.empty(nb + 16, dtype=torch.uint8, device="cuda")
        gb.synth_blocks(4, W, nb // gb.BLOCK_BYTES[4], SEED, 5)
        X = torch.randn(T * K, device="cuda")
        Y = torch.empty(T * N, device="cuda")
        f16 = os.environ.get("GB_GEMM_KIND", "") != "tf32"
        if f16:
            sb = gb.gemm_split_bytes(T, K)
            xh = torch.empty(sb, dtype=torch.uint8, device="cuda")
            xl = torch.empty(sb, dtype=torch.uint8, device="cuda")
            xi = torch.empty(T, device="cuda")
            gb.gemm_split(X, T, K, xh, xl, xi, stream=st.cuda_stream)
            run = lambda: gb.gemm_presplit(4, W, xh, xl, xi, Y, N, K, T, stream=st.cuda_stream)  # noqa: E731
        else:
            run = lambda: gb.gemm(4, W, X, Y, N, K, T, stream=st.cuda_stream)  # noqa: E731
        peak = bf16_peak() if f16 else peak_tf32
        for _ in range(3):
            run()
        e0.record(st)
        for _ in range(5):
            run()
        e1.record(st)
        e1.synchronize()
        g_ms = e0.elapsed_time(e1) / 5
        if gb.lib().gb_gemm_error(1) != 0:
            raise RuntimeError("gemm timeout")
        tf = 3 * 2.0 * N * K * T / (g_ms * 1e-3) / 1e12
        del W, X, Y
        flops = 2.0 * T * sum(r * cc for r, cc in _llama_layer_shapes()) * c["n_layers"]
        return {"metric": "prompt tokens/s (Llama-3.1-8B arch, Q4_K_M, 4096-token prompt, batch 1)",
                "value": round(T / (ms * 1e-3), 1), "unit": "tokens/s", "ms_per_prompt": round(ms, 2),
                "config": {"workload": f"llama3.1-8b-q4km-prefill, {T}-token prompt at position 0, 32 layers",
                           "chunk": min(T, 4096), "reps": reps, "warmup": 1,
                           "l2": "weights 4.9 GB and activations > 126 MB L2 per prompt"},
                "dtype": ("fp32-equivalent (weights dequantised to fp32, " +
                          ("3xF16 with power-of-two row scales" if f16 else "3xTF32") +
                          " tensor-core GEMMs, 3xTF32 attention)"),
                "layer_gemm_tflops_fp32_equiv": round(flops / (ms * 1e-3) / 1e12, 1),
                "e2e": {"value": round(T / e2e_s, 1), "unit": "tokens/s", "h2d_bytes_per_step": 4 * T,
                        "d2h_bytes_per_step": 8, "api": "gb_model_prefill_host (prompt in, next token out)"},
                "next_token": int(nxt),
                "roofline": {"bound": "tensor", "kernel": f"k_gemm<Q4_K> gate/up 14336x4096 at T={T}",
                             "achieved": round(tf, 1), "peak": round(peak, 1), "unit": "TFLOP/s",
                             "frac": round(tf / peak, 3),
                             "traffic": ncu_traffic("gemm_q4k_14336x4096_T4096.md"),
                             "fp32_equiv_tflops": round(tf / 3, 1), "ms": round(g_ms, 3),
                             "peak_kind": ("fp16 dense = the measured bf16 dense sustained rate" if f16 else
                                           "tf32 dense = half the measured bf16 dense sustained rate")}}
    finally:
        dm.close()


def _llama_layer_shapes():
    c = LLAMA8B
    H, kv, F = c["hidden_dim"], c["n_kv_heads"] * 128, c["ff_dim"]
    return [(H, H), (kv, H), (kv, H), (H, H), (F, H), (F, H), (H, F)]


def run_ours(args, rank, world, local_rank):
    import torch
    import guanaco_b200 as gb
    torch.cuda.set_device(local_rank)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    peak, peak_kind = peaks()
    K, W = args.steps, args.warmup
    c = LLAMA8B
    max_seq = CTX + 2 * (W + K) + 64
    # N > 1: tensor parallelism (one token stream, each GPU holds 1/N of the
    # weights and KV); the ranks add partial hidden vectors over NVLink
    dm = gb.DecodeModel(c["hidden_dim"], c["n_heads"], c["n_kv_heads"], c["n_layers"], c["ff_dim"],
                        c["vocab_size"], max_seq, tp_rank=rank, tp_world=world)
    if world > 1:
        dm.exchange_handles(dist)
    dm.synthesize(SEED)
    dm.fill_kv(CTX, SEED)
    st = torch.cuda.Stream()
    d_tok = torch.tensor([1], dtype=torch.int32, device="cuda")
    d_pos = torch.tensor([CTX], dtype=torch.int32, device="cuda")
    toks = torch.zeros(max(W, K) + 1, dtype=torch.int32, device="cuda")
    dm.generate(d_tok, d_pos, W, toks, stream=st.cuda_stream)
    st.synchronize()
    if dm.error() != 0:
        raise RuntimeError(f"decode error {dm.error()}")
    pos_timed0 = CTX + W

    with Clocks(local_rank) as clk:
        if dist:
            dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        dm.generate(d_tok, d_pos, K, toks, stream=st.cuda_stream)
        e1.record(st)
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
    t_ms = e0.elapsed_time(e1)
    if dist:
        tt = torch.tensor([t_ms], dtype=torch.float64, device="cuda")
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        t_ms = float(tt.item())
    if dm.error() != 0:
        raise RuntimeError(f"decode error {dm.error()}")
    timed_tokens = toks[:K].cpu().tolist()
    if args.decode_only:   # profiling runs: the timed decode steps only
        if dist:
            dist.barrier()
        dm.close()
        if dist:
            dist.destroy_process_group()
        if rank == 0:
            print(json.dumps({"decode_only": True, "ms_per_step": round(t_ms / K, 4)}), flush=True)
        return None
    tokens = K   # one token stream, whatever the number of GPUs
    value = tokens / (t_ms / 1e3)
    ms_per_step = t_ms / K

    # e2e: the host-buffer C-ABI call, token in / next token out per step
    pos = CTX + W + K
    tok = 1
    for _ in range(3):
        tok = dm.decode_host(tok, pos)
        pos += 1
    if dist:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(K):
        tok = dm.decode_host(tok, pos)
        pos += 1
    t_e2e = time.perf_counter() - t0
    if dist:
        tt = torch.tensor([t_e2e], dtype=torch.float64, device="cuda")
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        t_e2e = float(tt.item())
    e2e = K / t_e2e

    step_bytes = dm.step_bytes(pos_timed0 + K // 2)   # this rank's share
    if dist:
        sb = torch.tensor([step_bytes], dtype=torch.float64, device="cuda")
        dist.all_reduce(sb)
        step_bytes = float(sb.item())
    kernels, main = (None, None)
    if rank == 0:
        kernels, main = kernel_benchmarks(gb, torch, dm, peak)
    launches = dm.launches_per_step() * K + K   # + the feedback kernel per step
    if dist:
        dist.barrier()   # every rank is done with the peers' exchange buffers
    dm.close()
    tokens_check = None
    tiny = None
    if rank == 0 and world > 1:   # the tensor-parallel tokens against a one-GPU model
        ref_toks = one_gpu_tokens(gb, torch, max_seq, W, K)
        tokens_check = {"tokens_match": ref_toks == timed_tokens, "steps_compared": K,
                        "against": "one-GPU model of the same seeded weights and KV fill"}
    prefill = None
    if rank == 0 and world == 1 and not args.no_extra:
        tiny = tinyllama_decode(gb, torch)
        prefill = prefill_bench(gb, torch, tf32_peak())
        if not args.no_cpu_baseline:
            cores = os.cpu_count() or 1
            rate = cpu_reference_prefill_rate(cores)
            if rate:
                prefill["cpu_baseline"] = {
                    "value": round(rate, 3), "unit": "tokens/s", "cores": cores, "kind": "reference",
                    "sample": "reference forward() over a 32-token prompt (oracle/_ref) on one Llama-8B-width "
                              "layer plus the output head, head timed alone; rate = 32 / (32 x layer time)"}

    line = None
    if rank == 0:
        gbs, alg, t_launch = main
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            cores = os.cpu_count() or 1
            tt = cpu_reference_token_time(cores)
            if tt:
                cpu = {"value": round(1.0 / tt, 4), "unit": "tokens/s", "cores": cores, "kind": "reference",
                       "sample": "reference forward() (oracle/_ref) on the Llama-8B config at pos 4096: one "
                                 "layer + output head timed, head timed alone, token = head + 32 x layer; "
                                 "Q4_K matvec uses all cores, Q6_K is single-threaded in the reference"}
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "tokens/s", "n_gpus": world, "steps": K,
            "warmup": W, "ms_per_step": round(ms_per_step, 4), "higher_is_better": True,
            "scaling": "strong" if world > 1 else "weak",
            "vs_baseline": None,
            "dtype": "f32 (weights Q4_K/Q6_K codes; matvec x as three int8 limbs per 32-column sub-block, "
                     "24 significant bits as fp32; fp32 scales, accumulation, KV cache and attention)",
            "data": "synthetic (seeded random-init weights, ~N(0,1) KV fill)",
            "config": {"workload": "llama3.1-8b-q4km-decode (BASELINE config 4)", "global_batch": 1,
                       "seq_len": CTX, "parallelism": f"tp{world}" if world > 1 else "single",
                       "weights": "Q4_K + Q6_K(attn_v, ffn_down, output)", "kv": "fp32 head-major",
                       "l2": "weights 4.9 GB stream every step (> 126 MB L2); no flush needed",
                       "positions": [pos_timed0, pos_timed0 + K - 1],
                       "step_alg_bytes": round(step_bytes),
                       "step_hbm_frac": round(step_bytes / world / (t_ms / K * 1e-3) / 1e9 / peak, 3)},
            "e2e": {"value": round(e2e, 2), "unit": "tokens/s", "h2d_bytes_per_step": 8, "d2h_bytes_per_step": 8,
                    "api": "gb_model_decode_host (token, pos in; next token out)"},
            "gpu_launches": launches,
            "roofline": {"bound": "hbm", "kernel": "k_mvt Q4_K gate+up, one launch over 2 x 14336x4096 (the step's "
                                                   "largest launch share)", "achieved": round(gbs, 1),
                         "peak": peak, "unit": "GB/s", "frac": round(gbs / peak, 3), "traffic": ncu_traffic(),
                         "alg_bytes_per_launch": alg, "peak_kind": peak_kind},
            "kernels": kernels,
            "tokens": tokens_check,
            "config3": tiny,
            "prefill": prefill,
            "cpu_baseline": cpu,
            "clocks": clk.summary(),
        }
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    return line


def profile_kernel(name: str) -> None:
    """A few launches of one kernel on a case that fits an ncu capture
    (inputs larger than L2, a few hundred MB on the device): 3 warm-up
    launches, then 2 more.  Prints the per-launch time of the last two."""
    import torch
    import guanaco_b200 as gb
    torch.cuda.set_device(0)
    st = torch.cuda.Stream()
    sp = st.cuda_stream
    if name == "attn":
        nh, nkv, hd, ms, pos = 32, 8, 128, 8448, 8192
        copies = 3
        n = nkv * ms * hd
        kc = [torch.empty(n, dtype=torch.float32, device="cuda") for _ in range(copies)]
        vc = [torch.empty(n, dtype=torch.float32, device="cuda") for _ in range(copies)]
        for j in range(copies):
            gb.synth_normal(kc[j], n, SEED, 10 + j, stream=sp)
            gb.synth_normal(vc[j], n, SEED, 20 + j, stream=sp)
        q = torch.ones(nh * hd, dtype=torch.float32, device="cuda")
        k = torch.ones(nkv * hd, dtype=torch.float32, device="cuda")
        v = torch.ones(nkv * hd, dtype=torch.float32, device="cuda")
        cs = torch.empty(ms * hd, dtype=torch.float32, device="cuda")
        gb.rope_table(cs, ms, hd, stream=sp)
        ws = torch.zeros(gb.attn_workspace_bytes(nh, nkv, hd, ms), dtype=torch.uint8, device="cuda")
        d_pos = torch.tensor([pos], dtype=torch.int32, device="cuda")
        out = torch.empty(nh * hd, dtype=torch.float32, device="cuda")
        launch = lambda i: gb.attention_decode(q, k, v, kc[i % copies], vc[i % copies], cs, d_pos, nh, nkv, hd,  # noqa
                                               ms, out, ws, stream=sp)
    elif name == "prefill":   # whole prefills (launch lists): 1 warm-up + 2 timed
        c = LLAMA8B
        dm = gb.DecodeModel(c["hidden_dim"], c["n_heads"], c["n_kv_heads"], c["n_layers"], c["ff_dim"],
                            c["vocab_size"], PREFILL_T + 8)
        dm.synthesize(SEED)
        toks = torch.randint(0, c["vocab_size"], (PREFILL_T,), dtype=torch.int32,
                             generator=torch.Generator().manual_seed(SEED)).to("cuda")
        lg = torch.empty(c["vocab_size"], device="cuda")
        nx = torch.empty(1, dtype=torch.int32, device="cuda")
        dm.prefill(toks, PREFILL_T, 0, lg, nx, stream=sp)
        st.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        for _ in range(2):
            dm.prefill(toks, PREFILL_T, 0, lg, nx, stream=sp)
        e1.record(st)
        e1.synchronize()
        err = dm.error()
        dm.close()
        print(json.dumps({"kernel": name, "ms_per_prefill": round(e0.elapsed_time(e1) / 2, 2), "error": err}))
        return
    elif name == "pf_attn":   # prefill causal attention, 4096-token prompt at position 0
        nh, nkv, hd, T = 32, 8, 128, PREFILL_T
        n = nkv * T * hd
        kc = torch.empty(n, dtype=torch.float32, device="cuda")
        vc = torch.empty(n, dtype=torch.float32, device="cuda")
        q = torch.empty(T * nh * hd, dtype=torch.float32, device="cuda")
        gb.synth_normal(kc, n, SEED, 10, stream=sp)
        gb.synth_normal(vc, n, SEED, 20, stream=sp)
        gb.synth_normal(q, T * nh * hd, SEED, 30, stream=sp)
        out = torch.empty_like(q)
        launch = lambda i: gb.prefill_attention(q, kc, vc, out, T, 0, nh, nkv, hd, T, stream=sp)  # noqa: E731
    elif name in ("gemm_q4k", "gemm_q6k"):   # prefill GEMM at the 4096-token prompt
        dt, rows, cols = (4, 14336, 4096) if name == "gemm_q4k" else (5, 4096, 14336)
        T = PREFILL_T
        wb = gb.matrix_bytes(dt, rows, cols)
        W = torch.empty(wb + 16, dtype=torch.uint8, device="cuda")
        gb.synth_blocks(dt, W, wb // gb.BLOCK_BYTES[dt], SEED, 40, stream=sp)
        X = torch.empty(T * cols, dtype=torch.float32, device="cuda")
        gb.synth_normal(X, T * cols, SEED, 5, stream=sp)
        Y = torch.empty(T * rows, dtype=torch.float32, device="cuda")
        if os.environ.get("GB_GEMM_KIND", "") != "tf32":   # the GEMM launch alone on a split X
            sb = gb.gemm_split_bytes(T, cols)
            xh = torch.empty(sb, dtype=torch.uint8, device="cuda")
            xl = torch.empty(sb, dtype=torch.uint8, device="cuda")
            xi = torch.empty(T, dtype=torch.float32, device="cuda")
            gb.gemm_split(X, T, cols, xh, xl, xi, stream=sp)
            launch = lambda i: gb.gemm_presplit(dt, W, xh, xl, xi, Y, rows, cols, T, stream=sp)  # noqa: E731
        else:
            launch = lambda i: gb.gemm(dt, W, X, Y, rows, cols, T, stream=sp)  # noqa: E731
    elif name == "q4k_gu":   # gate + up in one launch, as in the decode step
        rows, cols, copies = 14336, 4096, 3
        wb = gb.matrix_bytes(4, rows, cols)
        bufs = [[torch.empty(wb + 16, dtype=torch.uint8, device="cuda") for _ in range(2)] for _ in range(copies)]
        for j, pair in enumerate(bufs):
            for i, b in enumerate(pair):
                gb.synth_blocks(4, b, wb // gb.BLOCK_BYTES[4], SEED, 60 + 2 * j + i, stream=sp)
        x = torch.empty(cols, dtype=torch.float32, device="cuda")
        gb.synth_normal(x, cols, SEED, 5, stream=sp)
        ys = [torch.empty(rows, dtype=torch.float32, device="cuda") for _ in range(2)]
        launch = lambda i: gb.matvec_group([4, 4], bufs[i % copies], [rows, rows], cols, x, ys, stream=sp)  # noqa
    else:
        dt, rows, cols, copies = {"q4k": (4, 14336, 4096, 6), "q6k": (5, 4096, 14336, 4),
                                  "q6k_head": (5, 128256, 4096, 1), "q8_0": (2, 14336, 4096, 4)}[name]
        wb = gb.matrix_bytes(dt, rows, cols)
        bufs = [torch.empty(wb + 16, dtype=torch.uint8, device="cuda") for _ in range(copies)]
        for j, b in enumerate(bufs):
            gb.synth_blocks(dt, b, wb // gb.BLOCK_BYTES[dt], SEED, 40 + j, stream=sp)
        x = torch.empty(cols, dtype=torch.float32, device="cuda")
        gb.synth_normal(x, cols, SEED, 5, stream=sp)
        y = torch.empty(rows, dtype=torch.float32, device="cuda")
        launch = lambda i: gb.matvec(dt, bufs[i % copies], rows, cols, x, y, stream=sp)  # noqa: E731
    for i in range(3):
        launch(i)
    st.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for i in range(3, 5):
        launch(i)
    e1.record(st)
    e1.synchronize()
    print(json.dumps({"kernel": name, "us_per_launch": round(e0.elapsed_time(e1) / 2 * 1e3, 2)}))


# ---------------------------------------------------------------- reference arm
def run_reference(args, rank, world):
    """The reference's own CPU implementation of the path (oracle/_ref: the
    reference C sources compiled unchanged) on the host cores, same metric.
    Each step is a bounded sample (see cpu_reference_token_time)."""
    if rank != 0:
        return None
    from oracle import oracle as O
    if not O.ref_available():
        return {"impl": "reference", "unavailable": "oracle/_ref/libref.so was not built"}
    cores = os.cpu_count() or 1
    for _ in range(max(0, min(args.warmup, 1))):
        cpu_reference_token_time(cores, reps=1)
    times = [cpu_reference_token_time(cores, reps=1) for _ in range(args.steps_ref)]
    tt = statistics.median(times)
    v = 1.0 / tt
    return {"metric": METRIC, "value": round(v, 4), "unit": "tokens/s", "n_gpus": world, "steps": len(times),
            "warmup": args.warmup, "ms_per_step": round(tt * 1e3, 1), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "impl": "reference",
            "config": {"workload": "llama3.1-8b-q4km-decode (BASELINE config 4)", "global_batch": 1,
                       "seq_len": CTX, "parallelism": "host threads"},
            "cpu_baseline": {"value": round(v, 4), "unit": "tokens/s", "cores": cores, "kind": "reference",
                             "sample": "per step: reference forward() with one Llama-8B layer + output head at "
                                       "pos 4096, output head timed alone; token = head + 32 x layer"},
            "e2e": {"value": round(v, 4), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extra", action="store_true", help="skip the config-3 (TinyLlama) and prefill lines")
    ap.add_argument("--decode-only", action="store_true",
                    help="run the warm-up and timed decode steps only (for ncu launch lists) and exit")
    ap.add_argument("--steps-ref", type=int, default=None, help="reference arm samples (default min(steps, 5))")
    ap.add_argument("--kernel", choices=["q4k", "q4k_gu", "q6k", "q6k_head", "q8_0", "attn", "pf_attn", "gemm_q4k",
                                         "gemm_q6k", "prefill"], default=None,
                    help="run only a few launches of one kernel (for ncu captures) and exit")
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == "ours":
        args.warmup = 3
    args.steps_ref = args.steps_ref or max(1, min(args.steps, 5))
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.kernel:
        return profile_kernel(args.kernel)
    if args.impl == "reference":
        line = run_reference(args, rank, world)
    else:
        line = run_ours(args, rank, world, local_rank)
    if rank == 0 and line is not None:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
