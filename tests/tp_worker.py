"""One rank of the tensor-parallel GPU check (launched by test_tp_gpu.py via
torch.distributed.run): builds the sharded engine on GPU LOCAL_RANK, runs the
prompt and a greedy continuation, and rank 0 compares tokens and logits with
an unsharded engine and the CPU oracle.  Prints TP_OK on success."""
import os
import sys
from pathlib import Path

import numpy as np
import torch
import torch.distributed as dist

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT / "inferno.jl_b200"))
sys.path.insert(0, str(ROOT / "oracle"))
from inferno_b200 import synth as S  # noqa: E402
from inferno_b200.model import Model  # noqa: E402


def main():
    name = sys.argv[1] if len(sys.argv) > 1 else "tiny-tp"
    n_steps = int(sys.argv[2]) if len(sys.argv) > 2 else 16
    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    dist.init_process_group("gloo")
    spec = S.CONFIGS[name]
    T = S.make_model(spec, seed=41)
    uid = [Model.tp_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(uid, src=0)
    torch.cuda.set_device(local)
    ok = True
    # 9 tokens: an 8-token chunk on the batched GEMV; 40 tokens: a 39-token
    # chunk on the tensor-core GEMM (dense models), then the last token and
    # the greedy continuation through the token path
    for plen in (9, 40):
        prompt = S.tokens(41, plen, spec.vocab)
        m = Model(spec, T, device=local, tp_rank=rank, tp_size=world, tp_uid=uid[0]) if plen == 9 else m
        m.reset()
        am, lg = m.forward(prompt, 0)
        out = m.decode_greedy(am, len(prompt), n_steps)
        if rank == 0:
            ref = Model(spec, T, device=local)
            am1, lg1 = ref.forward(prompt, 0)
            out1 = ref.decode_greedy(am1, len(prompt), n_steps)
            ref.close()
            import oracle as O
            orc = O.OracleModel(spec, T)
            amo, lgo = orc.forward(prompt, 0)
            rel = float(np.abs(lg - lg1).max() / np.abs(lg1).max())
            relo = float(np.abs(lg - lgo).max() / np.abs(lgo).max())
            print(f"tp={world} prompt {plen}: argmax {am} vs tp1 {am1} vs oracle {amo}; logits rel vs tp1 {rel:.2e}, "
                  f"vs oracle {relo:.2e}")
            print("tokens tp ", list(out))
            print("tokens tp1", list(out1))
            ok = ok and am == am1 == amo and list(out) == list(out1) and rel < 2e-3 and relo < 2e-3
    m.close()
    if rank == 0:
        print("TP_OK" if ok else "TP_MISMATCH", flush=True)
    dist.barrier()
    dist.destroy_process_group()
    sys.exit(0 if ok else 1)


if __name__ == "__main__":
    main()
