"""Per-kernel timeline of one decode frame (profiling tool).

`run` drives a batch of `--batch` requests (prompts of `--prompt` tokens,
teacher-forced codes) until every request decodes, then records one frame
with the library's launch trace (Q3T_KERNEL_TRACE: thread 0 of every CTA of
every talker / code-predictor kernel writes its grid id and %globaltimer
stamps) and writes the records to `--out`.  `summary` groups the records
by launch and prints, per kernel shape, the mean of:

* lag: the previous launch's last CTA exit -> this launch's first CTA past
  its dependency wait (the cost of a kernel boundary under programmatic
  dependent launch);
* post: first CTA past the wait -> last CTA exit (the launch's own critical
  path);
* for k_gemm, from the first wait release: X staged, MMAs done, split-K
  reduction barrier passed, epilogue done (each the latest CTA).

    python tts-rs_b200/ktrace.py run --batch 64 --prompt 16 --out frame.bin
    python tts-rs_b200/ktrace.py summary frame.bin
"""
import argparse
import os
import sys
import warnings

import numpy as np

KINDS = {1: "rmsnorm", 2: "gemm", 3: "attention", 4: "sampler"}
REC = np.dtype([("grid", "u8"), ("t", "u8", 7), ("kind", "i4"), ("cta", "i4"), ("n", "i4"), ("k", "i4")])


def run(args):
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path[:0] = [here]
    import q3t
    import synthetic as S
    cfg = S.TalkerConfig()
    model = q3t.Model(cfg, S.make_talker_weights(cfg, 0), kv_pages=args.kv_pages, max_active=args.batch)
    b = model.batch(max_active=args.batch, codec_mode=0, keep_output=0)
    H = cfg.talker.hidden
    for i in range(args.batch):
        g = np.random.default_rng([0, 77, 10000 + i])
        prompt = g.standard_normal((args.prompt, H), dtype=np.float32) * 0.5
        trailing = g.standard_normal((1, H), dtype=np.float32) * 0.5
        pad = g.standard_normal((H,), dtype=np.float32) * 0.5
        # long enough that no request retires before the traced frame
        codes = g.integers(0, 2048, size=(args.prompt * args.batch // 64 + args.settle + 100, 16), dtype=np.int64)
        b.submit(prompt, trailing, pad, codes.shape[0], forced=codes)
    # every prompt runs within prompt * batch / 64 + 2 steps (at least 64
    # prompt tokens ride in every talker pass); bounded either way
    for _ in range(args.prompt * args.batch // 64 + 8):
        st = b.step()
        if st["active"] == args.batch and st["prefill_tokens"] == 0:
            break
    for _ in range(args.settle):
        st = b.step()
    os.environ["Q3T_KERNEL_TRACE"] = args.out
    traced = b.step()
    del os.environ["Q3T_KERNEL_TRACE"]
    plain = b.step()
    b.close()
    model.close()
    print("traced frame:", traced)
    print("untraced frame:", plain)


def load(path):
    with open(path, "rb") as f:
        n, sz = np.frombuffer(f.read(8), np.int32)
        if sz != REC.itemsize:
            raise SystemExit(f"record size {sz} != {REC.itemsize}: trace from another build")
        return np.frombuffer(f.read(), REC, count=n)


def summary(args):
    r = load(args.trace)
    launches = []
    for g in np.unique(r["grid"]):
        x = r[r["grid"] == g]
        t = x["t"].astype(np.float64)
        launches.append(dict(kind=int(x["kind"][0]), n=int(x["n"][0]), k=int(x["k"][0]),
                             entry=t[:, 0].min(), wait=t[:, 1].min(), exit=t[:, 6].max(),
                             st=[t[:, j].max() for j in range(7)]))
    launches.sort(key=lambda d: d["entry"])
    rows, prev = {}, None
    for d in launches:
        key = KINDS.get(d["kind"], str(d["kind"])) + (f" N{d['n']} K{d['k']}" if d["kind"] == 2 else "")
        rel = lambda v: (v - d["wait"]) / 1e3
        row = [(d["wait"] - prev) / 1e3 if prev else 0.0, (d["exit"] - d["wait"]) / 1e3]
        row += [rel(d["st"][j]) for j in (2, 3, 4, 5)] if d["kind"] == 2 else [np.nan] * 4
        rows.setdefault(key, []).append(row)
        prev = d["exit"]
    span = (launches[-1]["exit"] - launches[0]["entry"]) / 1e3
    print(f"{len(launches)} launches, {span:.1f} us first entry -> last exit, {span / len(launches):.2f} us per launch")
    print(f"| kernel | launches | lag us | post us | X staged | MMA done | reduction | epilogue |")
    print("|---|---|---|---|---|---|---|---|")
    lag = post = 0.0
    for k, v in sorted(rows.items()):
        a = np.array(v)
        with warnings.catch_warnings():
            warnings.simplefilter("ignore", RuntimeWarning)  # all-NaN stage columns of non-GEMM kernels
            m = np.nanmean(a, 0)
        lag += a[:, 0].sum()
        post += a[:, 1].sum()
        extra = " | ".join("-" if np.isnan(x) else f"{x:.2f}" for x in m[2:])
        print(f"| {k} | {len(v)} | {m[0]:.2f} | {m[1]:.2f} | {extra} |")
    print(f"sum of lags {lag:.1f} us, sum of post-wait paths {post:.1f} us")


def main():
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    sub = ap.add_subparsers(dest="cmd", required=True)
    r = sub.add_parser("run")
    r.add_argument("--batch", type=int, default=64)
    r.add_argument("--prompt", type=int, default=16)
    r.add_argument("--settle", type=int, default=40, help="untraced decode frames before the traced one")
    r.add_argument("--kv-pages", type=int, default=8192)
    r.add_argument("--out", required=True)
    s = sub.add_parser("summary")
    s.add_argument("trace")
    args = ap.parse_args()
    run(args) if args.cmd == "run" else summary(args)


if __name__ == "__main__":
    main()
