"""Per-kernel benchmark of the hand-written sm_100a kernels at the shapes of the benchmark models.

    python -m meshtrain_b200.ops.kernel_bench [--only NAME[,NAME|PREFIX*]] [--iters N] [--json FILE]

Each case runs the kernel through the extension, timed with CUDA events on the
launching stream after warm-up (synchronised on both sides), and reports the
achieved rate against the roofline of its bound: FLOP/s against the measured
cuBLAS bf16 peak for tensor-core kernels, bytes/s against the measured copy
bandwidth for memory-bound kernels.  Peaks come from ``MEASURED_PEAKS.json`` at
the repository root when present (``bf16_tflops``, ``hbm_gbs``), else from the
values given on the command line.  Inputs smaller than twice the 126 MB L2
rotate over distinct copies, so repeats read HBM.  Cases named ``lib_*`` time
the torch/cuBLAS/cuDNN op the reference uses at the same shape.  The same
cases, run once each with ``--iters 1 --warmup 0``, are the small workloads
for ``ncu`` captures.
"""

from __future__ import annotations

import argparse
import json
import statistics
import threading
from pathlib import Path

import torch

from meshtrain_b200 import ops

ROOT = Path(__file__).resolve().parents[2]


def peaks(tflops: float, gbs: float) -> tuple[float, float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["bf16_tflops"]), float(d["hbm_gbs"]), "measured"
    return tflops, gbs, "given"


def _bf(*shape, scale=1.0):
    return (torch.randn(*shape, device="cuda") * scale).to(torch.bfloat16)


class SmClock:
    """Samples the SM clock (NVML) every 0.5 ms while a timed loop runs; median MHz."""

    def __init__(self, device: int):
        self.samples: list[int] = []
        self._stop = threading.Event()
        self._nvml = None
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nvml = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(device)
        except Exception:  # no NVML: clocks are reported as null
            self._nvml = None

    def _run(self):
        while not self._stop.is_set():
            self.samples.append(self._nvml.nvmlDeviceGetClockInfo(self._h, self._nvml.NVML_CLOCK_SM))
            self._stop.wait(0.0005)

    def __enter__(self):
        if self._nvml:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *exc):
        if self._nvml:
            self._stop.set()
            self._t.join()

    def median(self):
        return int(statistics.median(self.samples)) if self.samples else None


def time_us(fn, iters: int, warmup: int) -> tuple[float, int | None]:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with SmClock(torch.cuda.current_device()) as clk:
        a.record()
        for _ in range(iters):
            fn()
        b.record()
        torch.cuda.synchronize()
    return a.elapsed_time(b) / max(iters, 1) * 1e3, clk.median()


L2_BYTES = 126 * 1024 * 1024


def rotating(make, working_set_bytes: int):
    """Calls of ``make()``'s function over enough distinct input sets to exceed L2.

    A kernel whose inputs fit in the 126 MB L2 would otherwise read them from L2
    on every timed repeat and report more than HBM bandwidth.  ``make`` builds
    one independent set of inputs and returns its zero-argument function; the
    returned function cycles through ``ceil(2 * L2 / working set)`` of them.
    """
    n = max(1, -(-2 * L2_BYTES // max(1, working_set_bytes)))
    fns = [make() for _ in range(n)]
    state = [0]

    def fn():
        f = fns[state[0] % n]
        state[0] += 1
        return f()
    return fn


def cases():
    """name -> (setup() -> (fn, flops, bytes))."""
    out = {}
    T = 8192  # one microbatch of the 0.48B GPT: 4 sequences x 2048 tokens

    def gemm(M, N, K, epi):
        def setup():
            x, w = _bf(M, K), _bf(N, K, scale=0.02)
            b = _bf(N)
            res = _bf(M, N)
            if epi == "gelu":
                fn = lambda: ops.linear(x, w, b, gelu=True)  # noqa: E731
            elif epi == "resid":
                fn = lambda: ops.linear(x, w, b, residual=res)  # noqa: E731
            else:
                fn = lambda: ops.linear(x, w, b)  # noqa: E731
            return fn, 2.0 * M * N * K, 2 * (M * K + N * K + M * N)
        return setup

    def dgrad(M, N, K):
        def setup():
            dy, w = _bf(M, N), _bf(N, K, scale=0.02)
            return (lambda: ops.linear_dgrad(dy, w)), 2.0 * M * N * K, 2 * (M * N + N * K + M * K)
        return setup

    def wgrad(M, N, K):
        def setup():
            dy, x = _bf(M, N), _bf(M, K)
            acc, bg = torch.zeros(N, K, device="cuda"), torch.zeros(N, device="cuda")
            return (lambda: ops.linear_wgrad_(dy, x, acc, bg)), 2.0 * M * N * K, 2 * (M * N + M * K) + 8 * N * K
        return setup

    d, f = 1280, 5120
    out["gemm_qkv_fwd"] = gemm(T, 3 * d, d, "none")
    out["gemm_fc1_gelu_fwd"] = gemm(T, f, d, "gelu")
    out["gemm_fc1_plain_fwd"] = gemm(T, f, d, "none")
    out["gemm_fc2_resid_fwd"] = gemm(T, d, f, "resid")
    out["gemm_fc1_dgrad"] = dgrad(T, f, d)
    out["gemm_fc2_wgrad"] = wgrad(T, d, f)
    out["gemm_8192_cube"] = gemm(8192, 8192, 8192, "none")

    def attn(B, S, H, Hk, hd, bwd):
        def setup():
            q, k, v = _bf(B, S, H, hd), _bf(B, S, Hk, hd), _bf(B, S, Hk, hd)
            o, lse = ops.attention(q, k, v, causal=True)
            flops = 4.0 * B * H * S * S * hd / 2
            if not bwd:
                return (lambda: ops.attention(q, k, v, causal=True)), flops, 2 * (q.numel() * 2 + k.numel() * 2)
            do = _bf(B, S, H, hd)
            return (lambda: ops.attention_bwd(do, q, k, v, o, lse, causal=True)), 2.5 * flops, 2 * 8 * q.numel()
        return setup

    # sequence-length sweep at a fixed number of tokens x heads: the same FLOPs spread over
    # fewer, longer CTAs shows how much each CTA's fixed cost (prologue, epilogue) weighs
    for B_, S_ in ((16, 512), (1, 8192)):
        out[f"attn_fwd_hd64_s{S_}"] = attn(B_, S_, 20, 20, 64, False)
        out[f"attn_bwd_hd64_s{S_}"] = attn(B_, S_, 20, 20, 64, True)
    out["attn_fwd_hd64"] = attn(4, 2048, 20, 20, 64, False)
    out["attn_bwd_hd64"] = attn(4, 2048, 20, 20, 64, True)
    out["attn_fwd_hd128_gqa"] = attn(1, 4096, 32, 8, 128, False)
    out["attn_bwd_hd128_gqa"] = attn(1, 4096, 32, 8, 128, True)

    def norm(T, d, rms, bwd):
        nbytes = (4 if bwd else 2) * T * d * 2

        def make():
            x, g, b = _bf(T, d), _bf(d), _bf(d)
            dy, dres = _bf(T, d), _bf(T, d)
            dg, db = torch.zeros(d, device="cuda"), torch.zeros(d, device="cuda")
            if rms:
                _, r = ops.rmsnorm(x, g)
                return (lambda: ops.rmsnorm_bwd(dy, x, g, r, dres, dg)) if bwd else (lambda: ops.rmsnorm(x, g))
            _, m, r = ops.layernorm(x, g, b)
            return (lambda: ops.layernorm_bwd(dy, x, g, m, r, dres, dg, db)) if bwd else \
                (lambda: ops.layernorm(x, g, b))

        def setup():
            return rotating(make, nbytes), 0.0, nbytes
        return setup

    out["layernorm_fwd"] = norm(T, 1280, False, False)
    out["layernorm_bwd"] = norm(T, 1280, False, True)
    out["rmsnorm_bwd_d4096"] = norm(4096, 4096, True, True)

    def colsum(T, N):
        def make():
            dy, acc = _bf(T, N), torch.zeros(N, device="cuda")
            ext = ops.extension()
            return lambda: ext.colsum_(dy, acc)

        def setup():
            return rotating(make, T * N * 2), 0.0, T * N * 2
        return setup

    out["colsum_bias_grad"] = colsum(T, 5120)

    def ce(T, V, Vpad):
        def make():
            logits = _bf(T, Vpad)
            y = torch.randint(0, V, (T,), device="cuda")
            loss = torch.zeros((), device="cuda")
            return lambda: ops.cross_entropy_chunk_(logits, V, y, loss, 1.0, 1.0)

        def setup():
            return rotating(make, T * Vpad * 2), 0.0, 2 * T * Vpad * 2
        return setup

    out["cross_entropy_fwd_bwd"] = ce(2048, 50257, 50264)

    def adam(n):
        def setup():
            p, g = torch.randn(n, device="cuda"), torch.randn(n, device="cuda")
            m, v = torch.zeros(n, device="cuda"), torch.zeros(n, device="cuda")
            pb = torch.empty(n, device="cuda", dtype=torch.bfloat16)
            return (lambda: ops.adam_(p, g, m, v, pb, lr=1e-3, beta1=0.9, beta2=0.999, eps=1e-8, weight_decay=0.0,
                                      decoupled=False, step=1)), 0.0, n * (4 * 4 + 3 * 4 + 2)
        return setup

    out["adam_flat"] = adam(64 * 1024 * 1024)
    out.update(library_cases())
    return out


def library_cases():
    """The library ops the reference dispatches to, at the same shapes (``lib_`` prefix).

    The reference's transformer block runs ``nn.Linear`` (cuBLAS), ``F.gelu``,
    ``nn.LayerNorm`` and ``F.scaled_dot_product_attention(is_causal=True)``
    (models/tiny_transformer.py:36-49), and ``torch.optim.Adam``.  Each case
    here times that torch call the same way as the hand-written kernel's case
    of the same suffix, so the two rows compare directly.  Attention is timed
    with torch's default backend choice and with each backend forced
    (``_cudnn`` / ``_flash`` / ``_efficient`` suffixes); the backward cases time
    ``torch.autograd.grad`` on a retained graph, i.e. the backward kernels only.
    """
    import torch.nn.functional as F
    from torch.nn.attention import SDPBackend, sdpa_kernel

    out = {}
    T, d, f = 8192, 1280, 5120

    def linear(M, N, K, epi):
        def setup():
            x, w, b, res = _bf(M, K), _bf(N, K, scale=0.02), _bf(N), _bf(M, N)
            if epi == "gelu":
                fn = lambda: F.gelu(F.linear(x, w, b))  # noqa: E731
            elif epi == "resid":
                fn = lambda: res + F.linear(x, w, b)  # noqa: E731
            else:
                fn = lambda: F.linear(x, w, b)  # noqa: E731
            return fn, 2.0 * M * N * K, 2 * (M * K + N * K + M * N)
        return setup

    def dgrad(M, N, K):
        def setup():
            dy, w = _bf(M, N), _bf(N, K, scale=0.02)
            return (lambda: dy @ w), 2.0 * M * N * K, 2 * (M * N + N * K + M * K)
        return setup

    def wgrad(M, N, K):
        def setup():
            dy, x = _bf(M, N), _bf(M, K)
            acc = torch.zeros(N, K, device="cuda")
            return (lambda: acc.add_(dy.t() @ x)), 2.0 * M * N * K, 2 * (M * N + M * K) + 8 * N * K
        return setup

    out["lib_gemm_qkv_fwd"] = linear(T, 3 * d, d, "none")
    out["lib_gemm_fc1_gelu_fwd"] = linear(T, f, d, "gelu")
    out["lib_gemm_fc2_resid_fwd"] = linear(T, d, f, "resid")
    out["lib_gemm_fc1_dgrad"] = dgrad(T, f, d)
    out["lib_gemm_fc2_wgrad"] = wgrad(T, d, f)
    out["lib_gemm_8192_cube"] = linear(8192, 8192, 8192, "none")

    backends = {"": None, "_cudnn": SDPBackend.CUDNN_ATTENTION, "_flash": SDPBackend.FLASH_ATTENTION,
                "_efficient": SDPBackend.EFFICIENT_ATTENTION}

    def sdpa(B, S, H, Hk, hd, bwd, backend):
        def setup():
            q = _bf(B, H, S, hd).requires_grad_(bwd)
            k = _bf(B, Hk, S, hd).requires_grad_(bwd)
            v = _bf(B, Hk, S, hd).requires_grad_(bwd)
            gqa = H != Hk

            def fwd():
                if backend is None:
                    return F.scaled_dot_product_attention(q, k, v, is_causal=True, enable_gqa=gqa)
                with sdpa_kernel([backend]):
                    return F.scaled_dot_product_attention(q, k, v, is_causal=True, enable_gqa=gqa)

            flops = 4.0 * B * H * S * S * hd / 2
            if not bwd:
                return fwd, flops, 2 * (q.numel() * 2 + k.numel() * 2)
            o = fwd()
            do = _bf(B, H, S, hd)
            return (lambda: torch.autograd.grad(o, (q, k, v), do, retain_graph=True)), 2.5 * flops, 2 * 8 * q.numel()
        return setup

    for B_, S_ in ((16, 512), (1, 8192)):
        out[f"lib_attn_fwd_hd64_s{S_}"] = sdpa(B_, S_, 20, 20, 64, False, None)
        out[f"lib_attn_bwd_hd64_s{S_}"] = sdpa(B_, S_, 20, 20, 64, True, None)
    for suffix, backend in backends.items():
        out[f"lib_attn_fwd_hd64{suffix}"] = sdpa(4, 2048, 20, 20, 64, False, backend)
        out[f"lib_attn_bwd_hd64{suffix}"] = sdpa(4, 2048, 20, 20, 64, True, backend)
        out[f"lib_attn_fwd_hd128_gqa{suffix}"] = sdpa(1, 4096, 32, 8, 128, False, backend)
        out[f"lib_attn_bwd_hd128_gqa{suffix}"] = sdpa(1, 4096, 32, 8, 128, True, backend)

    def layernorm(bwd):
        nbytes = (4 if bwd else 2) * T * d * 2

        def make():
            x = _bf(T, d).requires_grad_(bwd)
            ln = torch.nn.LayerNorm(d, device="cuda", dtype=torch.bfloat16)
            if not bwd:
                return lambda: ln(x)
            y = ln(x)
            dy = _bf(T, d)
            return lambda: torch.autograd.grad(y, (x, ln.weight, ln.bias), dy, retain_graph=True)

        def setup():
            return rotating(make, nbytes), 0.0, nbytes
        return setup

    out["lib_layernorm_fwd"] = layernorm(False)
    out["lib_layernorm_bwd"] = layernorm(True)

    def ce(Tc, V):
        nbytes = 2 * Tc * V * 2

        def make():
            logits = _bf(Tc, V).requires_grad_(True)
            y = torch.randint(0, V, (Tc,), device="cuda")

            def fn():
                loss = F.cross_entropy(logits.float(), y)
                return torch.autograd.grad(loss, logits)
            return fn

        def setup():
            return rotating(make, nbytes), 0.0, nbytes
        return setup

    out["lib_cross_entropy_fwd_bwd"] = ce(2048, 50257)

    def adam(n):
        def setup():
            p = torch.randn(n, device="cuda").requires_grad_(True)
            p.grad = torch.randn(n, device="cuda")
            opt = torch.optim.Adam([p], lr=1e-3, fused=True)
            return opt.step, 0.0, n * (4 * 4 + 3 * 4)
        return setup

    out["lib_adam_flat"] = adam(64 * 1024 * 1024)
    return out


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--only", help="comma-separated case names")
    ap.add_argument("--iters", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--peak-tflops", type=float, default=1590.0)
    ap.add_argument("--peak-gbs", type=float, default=6650.0)
    ap.add_argument("--json")
    args = ap.parse_args(argv)
    if not torch.cuda.is_available():
        raise SystemExit("kernel_bench needs a CUDA GPU")
    ops.set_backend("custom")
    tf, gbs, src = peaks(args.peak_tflops, args.peak_gbs)
    all_cases = cases()
    if args.only:
        names = []
        for item in args.only.split(","):
            if item.endswith("*"):
                names += [n for n in all_cases if n.startswith(item[:-1])]
            else:
                names.append(item)
    else:
        names = list(all_cases)
    rows = []
    for name in names:
        try:
            fn, flops, nbytes = all_cases[name]()
            us, mhz = time_us(fn, args.iters, args.warmup)
        except RuntimeError as exc:  # a library backend that does not take this shape
            if not name.startswith("lib_"):
                raise
            row = {"kernel": name, "unavailable": str(exc).splitlines()[0][:200]}
            rows.append(row)
            print(json.dumps(row), flush=True)
            continue
        row = {"kernel": name, "us": round(us, 2), "sm_mhz": mhz}
        if flops:
            row["tflops"] = round(flops / us / 1e6, 1)
            row["frac_of_peak"] = round(flops / us / 1e6 / tf, 3)
        else:
            row["gbs"] = round(nbytes / us / 1e3, 1)
            row["frac_of_peak"] = round(nbytes / us / 1e3 / gbs, 3)
        rows.append(row)
        print(json.dumps(row), flush=True)
    status = ops.read_status(torch.cuda.current_device())
    summary = {"peaks": {"bf16_tflops": tf, "hbm_gbs": gbs, "source": src}, "rows": rows, "kernel_status": status,
               "gpu": torch.cuda.get_device_name(0)}
    if args.json:
        Path(args.json).write_text(json.dumps(summary, indent=2))
    return 0 if status == 0 else 1


if __name__ == "__main__":
    raise SystemExit(main())
