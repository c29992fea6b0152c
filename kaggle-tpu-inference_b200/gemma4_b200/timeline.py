"""Per-phase timeline of one decode step from the ``-DG4_TRACE`` build of the library.

Build the tracing library first (``python kaggle-tpu-inference_b200/gemma4_b200/build.py
--trace``), then::

    python kaggle-tpu-inference_b200/gemma4_b200/timeline.py --layers 6

runs a random model of the config-4 shapes with ``--layers`` layers on ``cuda:0``
(``--engine step`` or ``ops``), decodes ``--warm`` tokens, traces one more step and prints,
for every operator kind, the mean over layers of the per-CTA ``%globaltimer`` spans in
microseconds:

* start-skew   -- first to last CTA passing the phase start
* stage        -- phase start -> activations staged (step kernel)
* const+bar    -- -> constants landed and consumer barrier passed (step kernel)
* compute      -- -> prologue done (operator prologue + barrier)
* first-tile   -- prologue done -> first weight tile ready
* tiles        -- first tile ready -> last tile done
* straggle     -- median to last CTA finishing the phase
* gap          -- last CTA finishing -> first CTA starting the next phase
* span         -- phase start -> next phase start

Event slots per phase (trace id = 8 * layer + kind; the LM head is 8 * layers):
0 start, 1 staged, 2 constants + barrier, 3 prologue done, 4 first tile, 5 last tile,
6 finish, 7 the peer partials of an all-reduce received (world > 1: the prologues of
router+MLP and of qkv / the LM head; ``xchg-wait`` = 7 - 2).  Attention phases use 3 (q/k
prologue), 4 (key stages), 5 (partials published), 6 (merge, merging CTA only).  ``attn-s`` / ``attn-f`` rows: sliding / full
layers.
"""
import argparse
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))

KINDS = ["qkv", "attn", "oproj", "rmlp", "moeup", "moedn"]
ROWS = ["qkv", "attn-s", "attn-f", "oproj", "rmlp", "moeup", "moedn"]  # attention: sliding / full layers
TRACE_CTAS, TRACE_EVENTS, TRACE_LAUNCHES = 160, 8, 512


def phase_stats(buf, layers, full=()):
    """Per-phase medians over the traced CTAs, averaged over the layers of each row of
    ROWS (``full``: indices of the full-attention layers)."""
    import numpy as np

    b = buf.astype(np.int64)
    ncta = int((b[0, :, 0] > 0).sum())
    rows = [(k, b[8 * l + k][:ncta], l) for l in range(layers) for k in range(6)]
    rows.append((6, b[8 * layers][:ncta], layers))
    stats = {k: [] for k in ROWS}

    def med(x):
        return float(np.median(x)) / 1e3 if len(x) else 0.0

    for i, (k, e, layer) in enumerate(rows[:-1]):
        s0, e1, e2, e3, e4, e5, e6, e7 = (e[:, j] for j in range(8))
        ok = (s0 > 0) & (e6 >= s0)
        if not ok.any():
            continue
        nxt = rows[i + 1][1][:, 0]
        nstart = nxt[nxt > 0].min()
        m3 = (e3 > s0) & ok
        m4 = (e4 > 0) & m3
        m5 = (e5 > 0) & m4
        m12 = (e1 > 0) & (e2 > 0) & m3
        name = KINDS[k] if k != 1 else ("attn-f" if layer in full else "attn-s")
        stats[name].append((
            (s0[ok].max() - s0[ok].min()) / 1e3,
            med(e1[m12] - s0[m12]), med(e2[m12] - e1[m12]), med(e3[m12] - e2[m12]),
            med(e4[m4] - e3[m4]), med(e5[m5] - e4[m5]),
            (e6[ok].max() - np.median(e6[ok])) / 1e3,
            (nstart - e6[ok].max()) / 1e3,
            (nstart - s0[ok].min()) / 1e3,
            med(e7[m12 & (e7 >= e2)] - e2[m12 & (e7 >= e2)]),  # exchange wait (world > 1)
        ))
    t0 = b[b > 0].min()
    span = (b[8 * layers][:ncta, 6].max() - t0) / 1e3
    return ncta, span, {k: np.array(v).mean(0) for k, v in stats.items() if v}


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--layers", type=int, default=6)
    ap.add_argument("--warm", type=int, default=132, help="tokens decoded before the traced step")
    ap.add_argument("--pos", type=int, default=0,
                    help="trace the step at this position instead (jumps there; 0: after --warm tokens)")
    ap.add_argument("--max-len", type=int, default=32768)
    ap.add_argument("--engine", choices=["step", "ops"], default="step")
    ap.add_argument("--lib", default=os.path.join(HERE, "libg4b200_trace.so"))
    ap.add_argument("--save", default="", help="also write the raw event buffer (.npy, rank 0)")
    args = ap.parse_args()
    os.environ["G4B200_LIB"] = os.path.abspath(args.lib)

    import numpy as np
    import torch

    from gemma4_b200 import _native as N
    from gemma4_b200.config import make_config
    from gemma4_b200.engine import Engine
    from gemma4_b200.model import Mesh

    cfg = make_config(num_hidden_layers=args.layers)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank, local = int(os.environ.get("RANK", "0")), int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:  # under torchrun: every rank traces its own GPU, rank 0 prints
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    eng = Engine(None, max_len=args.max_len, cfg=cfg, random_seed=3, mesh=Mesh(rank, world, local),
                 engine=args.engine)
    eng.compile_all()
    m = eng.model
    prompt = list(range(100, 132))
    m.reset(prompt)
    if args.pos > 0:  # positions pos-2.. read tokens_out (their values do not change the time)
        m.ctrl[0] = args.pos - 2
        m.step(2)
    else:
        m.step(len(prompt) + args.warm)
    torch.cuda.synchronize()
    m.step(1)
    torch.cuda.synchronize()
    m.check_status()
    buf = np.zeros((TRACE_LAUNCHES, TRACE_CTAS, TRACE_EVENTS), np.uint64)
    N.check(N.lib().g4_trace_read(buf.ctypes.data, buf.nbytes), "g4_trace_read")
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
        if rank != 0:
            return 0
    if args.save:  # [launch id][CTA][event] globaltimer ns; launch id = 8 * layer + kind
        np.save(args.save, buf)
    full = [i for i, t in enumerate(cfg.layer_types) if t == "full_attention"]
    ncta, span, st = phase_stats(buf, args.layers, full)
    print(f"engine {args.engine}, {args.layers} layers, world {world} (rank 0 shown), {ncta} CTAs traced, "
          f"position {int(m.ctrl[0].item()) - 1}, step span {span:.1f} us")
    cols = ["start-skew", "stage", "const+bar", "compute", "first-tile", "tiles", "straggle", "gap", "span",
            "xchg-wait"]
    print("kind   " + " ".join(f"{c:>10s}" for c in cols))
    for k in ROWS:
        if k in st:
            print(f"{k:6s} " + " ".join(f"{x:10.1f}" for x in st[k]))
    if world > 1:  # the two all-reduces' waits, inside the consumers' prologues
        nl = {k: (len(full) if k == "attn-f" else args.layers - len(full) if k == "attn-s" else args.layers)
              for k in st}
        wait = sum(st[k][9] * nl[k] for k in st)
        total = sum(st[k][8] * nl[k] for k in st)
        print(f"exchange wait (median CTA) {wait:.1f} us per step = {100 * wait / total:.1f}% of the "
              f"summed phase spans ({total:.1f} us)")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
