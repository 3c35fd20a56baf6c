"""Greedy generation from a GGUF model file: generate_moe's command line
(crates/model/examples/generate_moe.rs) on the library's decode step.

    python -m styx_b200.generate MODEL.gguf --prompt 1,2,3 -n 32 [--ctx 4096]
                                 [--kv-page 512] [--experts-in-host] [--device 0]

Token ids in, token ids out (the reference example reads and prints ids the
same way when no tokenizer is given); prefill and decode rates are printed
like the reference's summary line.
"""
from __future__ import annotations

import argparse
import sys
import time


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("model")
    ap.add_argument("--prompt", required=True, help="comma-separated token ids")
    ap.add_argument("-n", "--n-predict", type=int, default=32)
    ap.add_argument("--ctx", type=int, default=4096, help="n_ctx_max: positions the KV caches may hold")
    ap.add_argument("--kv-page", type=int, default=512,
                    help="KV cache rows per page, grown on demand (moe.rs:501-503); 0 allocates --ctx rows at once")
    ap.add_argument("--experts-in-host", action="store_true",
                    help="expert tensors in pinned host memory, read in place")
    ap.add_argument("--device", type=int, default=0)
    args = ap.parse_args(argv)

    import torch

    from . import gguf as G
    torch.cuda.set_device(args.device)
    prompt = [int(t) for t in args.prompt.split(",") if t.strip()]
    g = G.Gguf.open(args.model)
    model, keep = G.load_decode_model(g, args.ctx, args.device, args.experts_in_host, kv_page=args.kv_page)
    g.close()
    t0 = time.perf_counter()
    for t in prompt:
        model.forward_token(t)
    out = [int(model.next.item())]
    t1 = time.perf_counter()
    for _ in range(1, args.n_predict):
        model.forward_token(out[-1])
        out.append(int(model.next.item()))
    t2 = time.perf_counter()
    model.moe.ctx.check_device_error()
    print(",".join(str(t) for t in out))
    print(f"prefill {len(prompt) / (t1 - t0):.1f} tok/s, decode {(args.n_predict - 1) / max(t2 - t1, 1e-9):.1f} tok/s",
          file=sys.stderr)
    del keep
    return 0


if __name__ == "__main__":
    sys.exit(main())
