"""Timings of single operators and of the decoder layer on one GPU.

    python -m llama2_b200.microbench {gemm,attention,paged,paged_step,paged_prefill,fp8,pv,swiglu,unpad,rope,layer} [--iters N]

Each prints one line per shape. Kernels are timed with CUDA events on the
current stream; ``gemm`` times back-to-back launches of the products of
more than 128 rows (compute-bound, L2 irrelevant) and flushed launches of
the decode-sized ones (at most 128 rows: bound by reading B, whose 34-180 MB
would otherwise sit in L2 between launches), next to ``torch.matmul`` on the
same operands (cuBLAS, for reference); the others flush L2 before every
timed launch (write a 512 MB buffer, then read another, outside the timed
window). Inputs are seeded
random tensors of the 7B shapes.
"""
from __future__ import annotations

import argparse

import torch

from . import capi, ops

_FLUSH = {}


def _flush():
    if "w" not in _FLUSH:
        _FLUSH["w"] = torch.empty(512 << 20 >> 2, device="cuda")
        _FLUSH["r"] = torch.ones(512 << 20 >> 2, device="cuda")
    _FLUSH["w"].zero_()
    _FLUSH["r"].sum()


def time_ms(fn, iters: int, flush: bool = True) -> float:
    """Mean milliseconds of fn() over iters launches (after 3 untimed ones)."""
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    if not flush:
        a, z = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(iters):
            fn()
        z.record()
        torch.cuda.synchronize()
        return a.elapsed_time(z) / iters
    total = 0.0
    for _ in range(iters):
        _flush()
        a, z = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        z.record()
        torch.cuda.synchronize()
        total += a.elapsed_time(z)
    return total / iters


def bench_gemm(iters, shape=None):
    shapes = [(4096, 4096, 4096), (8192, 8192, 8192), (16384, 12288, 4096), (16384, 4096, 4096),
              (64, 12288, 4096), (64, 4096, 4096), (64, 22016, 4096), (64, 4096, 11008), (1, 12288, 4096)]
    for (m, n, k) in ([shape] if shape else shapes):
        for trans_b in ((0,) if shape else (0, 1)):
            a = torch.randn(m, k, device="cuda", dtype=torch.bfloat16)
            b = (torch.randn(n, k, device="cuda", dtype=torch.bfloat16) if trans_b
                 else torch.randn(k, n, device="cuda", dtype=torch.bfloat16))
            c = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
            ours = lambda: capi.call("l2k_linear", 0, trans_b, m, n, k, a.data_ptr(), k, b.data_ptr(), b.stride(0),
                                     c.data_ptr(), n, 0, None, None, None, capi.L2K_BF16,
                                     torch.cuda.current_stream().cuda_stream)
            ref = lambda: torch.matmul(a, b.t() if trans_b else b, out=c)
            flush = m <= 128
            t1, t2 = time_ms(ours, iters, flush=flush), time_ms(ref, iters, flush=flush)
            fl = 2.0 * m * n * k
            if flush:  # bytes of A, B and C per launch
                nb = 2.0 * (m * k + k * n + m * n)
                print(f"gemm bf16 m={m} n={n} k={k} trans_b={trans_b} (L2 flushed): {t1 * 1e3:.1f} us "
                      f"{nb / t1 / 1e6:.1f} GB/s | torch.matmul {t2 * 1e3:.1f} us {nb / t2 / 1e6:.1f} GB/s")
            else:
                print(f"gemm bf16 m={m} n={n} k={k} trans_b={trans_b}: {t1 * 1e3:.1f} us {fl / t1 / 1e9:.1f} TF/s | "
                      f"torch.matmul {t2 * 1e3:.1f} us {fl / t2 / 1e9:.1f} TF/s")


def bench_attention(iters):
    h, s, hd = 32, 4096, 128
    for dt in (torch.float32, torch.bfloat16):
        for b in (1, 16, 64):
            q = torch.randn(b, h, 1, hd, device="cuda").to(dt)
            k = torch.randn(b, h, s, hd, device="cuda").to(dt)
            v = torch.randn(b, h, s, hd, device="cuda").to(dt)
            lens = torch.randint(1, s, (b,), generator=torch.Generator().manual_seed(1))
            kv = lens.to(torch.uint32).cuda()
            mx = torch.tensor([int(lens.max())], dtype=torch.uint32, device="cuda")
            qk = torch.empty(b, h, 1, s, device="cuda", dtype=dt)
            out = torch.empty(b, h, 1, hd, device="cuda", dtype=dt)
            es = q.element_size()
            keys = int(lens.sum())
            for name, fn, nbytes in (
                    ("scores", lambda: ops.decode_attention_scores(q, k, kv, mx, qk),
                     keys * h * hd * es + b * h * int(mx) * es),
                    ("scores+P.V", lambda: ops.decode_attention(q, k, v, kv, mx, qk, out),
                     2 * keys * h * hd * es + b * h * int(mx) * es)):
                ms = time_ms(fn, iters)
                print(f"decode {name} {dt} b={b}: {ms * 1e3:.1f} us {nbytes / ms / 1e6:.1f} GB/s")


def bench_paged(iters):
    """Fused decode attention over a paged pool (shuffled block table) next
    to the same attention over the contiguous cache."""
    h, s, hd = 32, 4096, 128
    for dt in (torch.float32, torch.bfloat16):
        rows = ops.paged_block_rows(hd, dt)
        max_pages = s // rows
        for b in (1, 64):
            q = torch.randn(b, h, 1, hd, device="cuda").to(dt)
            k = torch.randn(b, h, s, hd, device="cuda").to(dt)
            v = torch.randn(b, h, s, hd, device="cuda").to(dt)
            perm = torch.randperm(b * max_pages, generator=torch.Generator().manual_seed(2))
            table = perm.view(b, max_pages).to(torch.int32).cuda()
            kp = torch.empty(b * max_pages, h, rows, hd, device="cuda", dtype=dt)
            vp = torch.empty_like(kp)
            kp[perm] = k.view(b, h, max_pages, rows, hd).transpose(1, 2).reshape(b * max_pages, h, rows, hd)
            vp[perm] = v.view(b, h, max_pages, rows, hd).transpose(1, 2).reshape(b * max_pages, h, rows, hd)
            lens = torch.randint(1, s, (b,), generator=torch.Generator().manual_seed(1))
            kv = lens.to(torch.uint32).cuda()
            mx = torch.tensor([int(lens.max())], dtype=torch.uint32, device="cuda")
            qk = torch.empty(b, h, 1, s, device="cuda", dtype=dt)
            out = torch.empty(b, h, 1, hd, device="cuda", dtype=dt)
            es = q.element_size()
            nbytes = 2 * int(lens.sum()) * h * hd * es + b * h * int(mx) * es
            t1 = time_ms(lambda: ops.decode_attention(q, k, v, kv, mx, qk, out), iters)
            t2 = time_ms(lambda: ops.decode_attention_paged(q, kp, vp, table, kv, mx, qk, out), iters)
            print(f"decode attention {dt} b={b}: contiguous {t1 * 1e3:.1f} us {nbytes / t1 / 1e6:.1f} GB/s | "
                  f"paged ({rows}-row pages) {t2 * 1e3:.1f} us {nbytes / t2 / 1e6:.1f} GB/s")
            del k, v, kp, vp


def bench_paged_step(iters):
    """The one-launch decode step (7B dims) over paged caches (shuffled block
    table) next to the same step over the contiguous caches."""
    h, s, hd, dim, hidden, vocab = 32, 4096, 128, 4096, 11008, 32000
    for dt in (torch.float32, torch.bfloat16):
        rows = ops.paged_block_rows(hd, dt)
        max_pages = s // rows
        b = 64
        g = torch.Generator(device="cuda")
        g.manual_seed(5)
        k = torch.randn(b, h, s, hd, device="cuda", generator=g).to(dt)
        v = torch.randn(b, h, s, hd, device="cuda", generator=g).to(dt)
        perm = torch.randperm(b * max_pages, generator=torch.Generator().manual_seed(2))
        table = perm.view(b, max_pages).to(torch.int32).cuda()
        kp = torch.empty(b * max_pages, h, rows, hd, device="cuda", dtype=dt)
        vp = torch.empty_like(kp)
        kp[perm] = k.view(b, h, max_pages, rows, hd).transpose(1, 2).reshape(b * max_pages, h, rows, hd)
        vp[perm] = v.view(b, h, max_pages, rows, hd).transpose(1, 2).reshape(b * max_pages, h, rows, hd)
        lens = torch.randint(1, s - 1, (b,), generator=torch.Generator().manual_seed(1))
        kv0 = lens.to(torch.uint32).cuda()
        kv = kv0.clone()
        base = dict(q_lens=torch.ones(b, dtype=torch.uint32, device="cuda"), kv_lens=kv,
                    max_lens=torch.zeros(2, dtype=torch.uint32, device="cuda"),
                    input_ids=torch.randint(0, vocab, (b,), dtype=torch.int32, device="cuda"),
                    embed_table=(torch.randn(vocab, dim, device="cuda", generator=g) * 0.02).to(dt),
                    norm_weight=torch.ones(dim, device="cuda", dtype=dt),
                    x=torch.empty(b, dim, device="cuda", dtype=dt), normed=torch.empty(b, dim, device="cuda", dtype=dt),
                    qkv=torch.randn(b, 3 * dim, device="cuda", generator=g).to(dt),
                    is_done=torch.zeros(b, dtype=torch.uint8, device="cuda"),
                    q=torch.empty(b, h, 1, hd, device="cuda", dtype=dt),
                    qk=torch.empty(b, h, 1, s, device="cuda", dtype=dt),
                    gate_up=torch.randn(b, 2 * hidden, device="cuda", generator=g).to(dt),
                    ffn_out=torch.empty(b, hidden, device="cuda", dtype=dt),
                    workspace=ops.decode_step_workspace(torch.device("cuda")), pairing=1)
        es = torch.finfo(dt).bits // 8
        nbytes = (int(lens.sum()) + b) * h * hd * es + b * h * s * es  # K rows read, score rows written

        def contiguous():
            kv.copy_(kv0)
            ops.decode_step(**base, k_cache=k, v_cache=v)

        def paged():
            kv.copy_(kv0)
            ops.decode_step_paged(**base, k_pages=kp, v_pages=vp, block_table=table)

        t1, t2 = time_ms(contiguous, iters), time_ms(paged, iters)
        print(f"decode step {dt} b={b}: contiguous {t1 * 1e3:.1f} us {nbytes / t1 / 1e6:.1f} GB/s | "
              f"paged ({rows}-row pages) {t2 * 1e3:.1f} us {nbytes / t2 / 1e6:.1f} GB/s")
        del k, v, kp, vp


def bench_paged_prefill(iters):
    """Prefill attention over paged K/V caches (64-row pages of 7B heads,
    shuffled block table) next to the contiguous operators: the tcgen05
    scores (8 x 2048 causal rows, bf16) and the tcgen05 P.V."""
    b, h, qc, hd = 8, 32, 2048, 128
    dt = torch.bfloat16
    rows = 64
    max_pages = qc // rows
    g = torch.Generator(device="cuda")
    g.manual_seed(3)
    q = torch.randn(b, h, qc, hd, device="cuda", generator=g).to(dt)
    k = torch.randn(b, h, qc, hd, device="cuda", generator=g).to(dt)
    v = torch.randn(b, h, qc, hd, device="cuda", generator=g).to(dt)
    perm = torch.randperm(b * max_pages, generator=torch.Generator().manual_seed(2))
    table = perm.view(b, max_pages).to(torch.int32).cuda()
    kp = torch.empty(b * max_pages, h, rows, hd, device="cuda", dtype=dt)
    vp = torch.empty_like(kp)
    kp[perm] = k.view(b, h, max_pages, rows, hd).transpose(1, 2).reshape(b * max_pages, h, rows, hd)
    vp[perm] = v.view(b, h, max_pages, rows, hd).transpose(1, 2).reshape(b * max_pages, h, rows, hd)
    ql = torch.full((b,), qc, dtype=torch.uint32, device="cuda")
    kl = torch.full((b,), qc, dtype=torch.uint32, device="cuda")
    qk = torch.empty(b, h, qc, qc, device="cuda", dtype=dt)
    out = torch.empty(b, h, qc, hd, device="cuda", dtype=dt)
    es = 2
    score_bytes = (2 * b * h * qc * hd + b * h * qc * qc) * es  # q, K, P
    pv_bytes = (b * h * qc * qc + 2 * b * h * qc * hd) * es     # P, V, output
    for name, fn_c, fn_p, nb in (
            ("scores", lambda: ops.prefill_attention_scores(q, k, ql, kl, qc, qc, qk),
             lambda: ops.prefill_attention_scores_paged(q, kp, table, ql, kl, qc, qc, qk), score_bytes),
            ("P.V", lambda: ops.launch_attention_qkv(qk, v, out, qc, qc),
             lambda: ops.launch_attention_qkv_paged(qk, vp, table, kl, out, qc, qc), pv_bytes)):
        t1, t2 = time_ms(fn_c, iters), time_ms(fn_p, iters)
        print(f"prefill {name} bf16 8 x 2048: contiguous {t1 * 1e3:.1f} us {nb / t1 / 1e6:.1f} GB/s | "
              f"paged (64-row pages) {t2 * 1e3:.1f} us {nb / t2 / 1e6:.1f} GB/s")


def bench_fp8(iters, batch=None):
    """Fused decode attention over fp8 (e4m3) caches next to bf16 caches of
    the same shape (7B heads, 4096-position caches, seeded lengths)."""
    h, s, hd = 32, 4096, 128
    for b in ([batch] if batch else (1, 16, 64)):
        q = torch.randn(b, h, 1, hd, device="cuda").to(torch.bfloat16)
        k16 = torch.randn(b, h, s, hd, device="cuda").to(torch.bfloat16)
        v16 = torch.randn(b, h, s, hd, device="cuda").to(torch.bfloat16)
        k8 = (k16.float() / 0.25).to(torch.float8_e4m3fn).view(torch.uint8)
        v8 = (v16.float() / 0.25).to(torch.float8_e4m3fn).view(torch.uint8)
        lens = torch.randint(1, s, (b,), generator=torch.Generator().manual_seed(1))
        kv = lens.to(torch.uint32).cuda()
        mx = torch.tensor([int(lens.max())], dtype=torch.uint32, device="cuda")
        qk = torch.empty(b, h, 1, s, device="cuda", dtype=torch.bfloat16)
        out = torch.empty(b, h, 1, hd, device="cuda", dtype=torch.bfloat16)
        keys = int(lens.sum())
        n16 = 2 * keys * h * hd * 2 + b * h * int(mx) * 2
        n8 = 2 * keys * h * hd + b * h * int(mx) * 2
        t16 = time_ms(lambda: ops.decode_attention(q, k16, v16, kv, mx, qk, out), iters)
        t8 = time_ms(lambda: ops.decode_attention_fp8(q, k8, v8, 0.25, 0.25, kv, mx, qk, out), iters)
        print(f"decode attention b={b}: bf16 caches {t16 * 1e3:.1f} us {n16 / t16 / 1e6:.1f} GB/s | "
              f"fp8 caches {t8 * 1e3:.1f} us {n8 / t8 / 1e6:.1f} GB/s ({t16 / t8:.2f}x)")
        del k16, v16, k8, v8


def bench_pv(iters):
    b, h, qc, s, hd = 8, 32, 2048, 2048, 128
    qk = torch.rand(b, h, qc, s, device="cuda", dtype=torch.bfloat16)
    v = torch.randn(b, h, s, hd, device="cuda", dtype=torch.bfloat16)
    out = torch.empty(b, h, qc, hd, device="cuda", dtype=torch.bfloat16)
    ms = time_ms(lambda: ops.launch_attention_qkv(qk, v, out, qc, s), iters)
    nbytes = (qk.numel() + v.numel() + out.numel()) * 2
    print(f"P.V bf16 {b}x{h}x{qc}x{s}: {ms * 1e3:.1f} us {nbytes / ms / 1e6:.1f} GB/s "
          f"{2 * b * h * qc * s * hd / ms / 1e9:.1f} TF/s")


def bench_swiglu(iters):
    for (t, dt) in ((16384, torch.bfloat16), (16384, torch.float32), (64, torch.bfloat16)):
        f = 11008
        inp = torch.randn(t, 2 * f, device="cuda").to(dt)
        out = torch.empty(t, f, device="cuda", dtype=dt)
        ms = time_ms(lambda: ops.launch_swiglu(inp, out), iters)
        nbytes = (inp.numel() + out.numel()) * inp.element_size()
        print(f"swiglu {dt} {t} x {f}: {ms * 1e3:.1f} us {nbytes / ms / 1e6:.1f} GB/s")


def bench_unpad(iters):
    b, h, qc, hd = 8, 32, 2048, 128
    qkv = torch.randn(b, h, qc, hd, device="cuda", dtype=torch.bfloat16)
    idx = torch.arange(b * qc, dtype=torch.int32, device="cuda")
    out = torch.empty(b * qc, h * hd, device="cuda", dtype=torch.bfloat16)
    ms = time_ms(lambda: ops.launch_fused_transpose_unpad(b * qc, qkv, idx, out), iters)
    print(f"transpose+unpad bf16 {b * qc} tokens: {ms * 1e3:.1f} us {2 * qkv.numel() * 2 / ms / 1e6:.1f} GB/s")


def bench_rope(iters):
    b, qc, h, hd = 8, 2048, 32, 128
    d, t = h * hd, b * qc
    for dt in (torch.bfloat16, torch.float32):
        inp = torch.randn(t, 3 * d, device="cuda").to(dt)
        lens = torch.full((b,), qc, dtype=torch.int32, device="cuda")
        idx = torch.arange(t, dtype=torch.int32, device="cuda")
        q = torch.empty(b, h, qc, hd, device="cuda", dtype=dt)
        k = torch.empty(b, h, qc, hd, device="cuda", dtype=dt)
        v = torch.empty(b, h, qc, hd, device="cuda", dtype=dt)
        ms = time_ms(lambda: ops.launch_fused_pad_reshape_transpose_rope_kvcache_llama2(inp, lens, lens, idx, q, k, v),
                     iters)
        print(f"prefill RoPE + KV append {dt} {t} tokens: {ms * 1e3:.1f} us "
              f"{2 * inp.numel() * inp.element_size() / ms / 1e6:.1f} GB/s")


def bench_layer(iters):
    from .layer import DecoderLayer
    for (b, dt, fuse) in ((64, torch.bfloat16, True), (64, torch.bfloat16, False), (1, torch.bfloat16, True),
                          (64, torch.float32, True)):
        layer = DecoderLayer(4096, 32, 32, 11008, 4096, b, dtype=dt, seed=0, fuse_epilogues=fuse)
        x = torch.randn(b, 4096, device="cuda").to(dt)
        q_lens = torch.ones(b, dtype=torch.uint32, device="cuda")
        lens = torch.randint(1, 4095, (b,), generator=torch.Generator().manual_seed(0))
        kv = lens.to(torch.uint32).cuda()
        max_lens = torch.zeros(2, dtype=torch.uint32, device="cuda")
        ops.launch_update_q_kv_lens(q_lens, kv, max_lens[0:1], max_lens[1:2])
        is_done = torch.zeros(b, dtype=torch.uint8, device="cuda")
        pending = torch.randn(b, 4096, device="cuda").to(dt)
        graph = layer.capture_decode(x, pending, kv, max_lens[1:2], is_done)
        ms = time_ms(graph.replay, iters)
        es = 2 if dt != torch.float32 else 4
        wbytes = sum(t.numel() for t in layer.weights().values()) * es
        kvb = 2 * int((lens + 1).sum()) * 4096 * es
        print(f"7B decoder layer decode step {dt} b={b} ({layer.launches_per_step()} launches): "
              f"{ms * 1e3:.1f} us; weights {wbytes / 1e6:.0f} MB + "
              f"K/V {kvb / 1e6:.0f} MB -> {(wbytes + kvb) / ms / 1e6:.0f} GB/s")
        del layer, graph
    # prefill pass of 8 prompts x 2048 new tokens (16384 token rows)
    b, qc = 8, 2048
    t = b * qc
    for fuse in (True, False):
        layer = DecoderLayer(4096, 32, 32, 11008, qc, b, dtype=torch.bfloat16, seed=0, fuse_epilogues=fuse)
        x = torch.randn(t, 4096, device="cuda").to(torch.bfloat16)
        q_lens = torch.full((b,), qc, dtype=torch.uint32, device="cuda")
        unpad = torch.zeros(b, qc, dtype=torch.uint32, device="cuda")
        offsets = torch.zeros(b, dtype=torch.uint32, device="cuda")
        ops.launch_build_padding_index_maps(t, q_lens, unpad, offsets)
        ms = time_ms(lambda: layer.prefill(x, None, q_lens, q_lens, qc, qc, unpad), iters)
        print(f"7B decoder layer prefill bf16 {t} tokens ({layer.launches_per_prefill(t)} launches): "
              f"{ms * 1e3:.1f} us, {t / ms / 1e3:.2f} M tokens/s")
        del layer


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("what", choices=["gemm", "attention", "paged", "paged_step", "paged_prefill", "fp8", "pv", "swiglu", "unpad",
                                        "rope", "layer"])
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--shape", default="", help="gemm: one M,N,K product (B stored K x N) instead of the set")
    ap.add_argument("--batch", type=int, default=0, help="fp8: one batch size instead of the set")
    args = ap.parse_args()
    torch.manual_seed(0)
    if args.what == "gemm":
        bench_gemm(args.iters, tuple(int(x) for x in args.shape.split(",")) if args.shape else None)
    elif args.what == "fp8":
        bench_fp8(args.iters, args.batch or None)
    else:
        globals()["bench_" + args.what](args.iters)


if __name__ == "__main__":
    main()
