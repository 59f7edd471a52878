"""One rank of the expert-parallel GPU test (launched by test_ep.py through
torch.distributed.run).  Each rank holds E/world experts of an oracle-generated
layer, runs the EP forward on its own tokens (eagerly and from a CUDA graph),
and rank 0 checks every rank's output bit for bit against a single-GPU context
holding all experts, also after the experts are placed on the ranks by a
permutation.  Exit status 0 = pass."""
import datetime
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
sys.path.insert(0, os.path.join(ROOT, "project-obsidian_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
import obsmoe  # noqa: E402
import oracle as O  # noqa: E402

E, H, I, K, SEED = 16, 2048, 256, 4, 7


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=60))
    L = O.synth_layer(SEED, 0, E=E, H=H, I=I, K=K)
    Ts = [37, 0, 130, 5][:world] if world <= 4 else [16 * (r + 1) for r in range(world)]
    T = Ts[rank]
    shape = obsmoe.MoeShape(H, I, E, K, n_layers=1, max_tokens=160, ep_world=world, ep_rank=rank)
    ctx = obsmoe.MoeContext(shape, local)
    ctx.load_layer(0, L)
    handles = [None] * world
    dist.all_gather_object(handles, ctx.ep_handle())
    ctx.ep_connect(handles)

    x = O.synth_x(SEED, 0, T, H, row0=1000 * rank)
    xd = torch.from_numpy(x.view(np.int16)).cuda()
    res = torch.from_numpy(O.synth_x(SEED + 1, 0, T, H, row0=1000 * rank).view(np.int16)).cuda()
    outs = []
    for rep in range(3):  # repeated forwards: the epochs advance
        out = torch.full((max(T, 1), H), -1, dtype=torch.int16, device="cuda")
        ctx.moe_forward(0, xd, out, T, residual=res if rep == 2 else None)
        torch.cuda.synchronize()
        outs.append(out[:T].cpu().numpy().view(np.uint16).copy())
    ctx.check_device()
    # the same forward captured in a CUDA graph, replayed twice
    gout = torch.full((max(T, 1), H), -1, dtype=torch.int16, device="cuda")
    cap = torch.cuda.Stream()
    cap.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(cap):
        with torch.cuda.graph(g, stream=cap):
            ctx.moe_forward(0, xd, gout, T, stream=cap)
    torch.cuda.current_stream().wait_stream(cap)
    dist.barrier()
    for _ in range(2):
        gout.fill_(-1)
        g.replay()
        torch.cuda.synchronize()
        outs.append(gout[:T].cpu().numpy().view(np.uint16).copy())
        dist.barrier()
    del g
    ctx.check_device()
    # another expert placement (the same seeded permutation on every rank): every rank refuses
    # the forward until the layer is loaded again, then the output is the same bits
    perm = [int(e) for e in np.random.default_rng(5).permutation(E)]
    ctx.ep_set_placement(0, perm)
    ok_local = ctx.ep_get_placement(0) == perm
    try:
        ctx.moe_forward(0, xd, out, T)
        ok_local = False
    except obsmoe.ObsError:
        pass
    ctx.load_layer(0, L)
    dist.barrier()
    for rep in range(2):
        out = torch.full((max(T, 1), H), -1, dtype=torch.int16, device="cuda")
        ctx.moe_forward(0, xd, out, T)
        torch.cuda.synchronize()
        outs.append(out[:T].cpu().numpy().view(np.uint16).copy())
        try:  # every rank checks and goes on, so the ranks stay in step
            ctx.check_device()
        except obsmoe.ObsError as err:
            print(f"rank {rank}: forward {rep} after the placement: {err}", flush=True)
            ok_local = False
        dist.barrier()
    print(f"rank {rank}: placement set, refused before reload, read back, device clean: {ok_local}", flush=True)

    gathered = [None] * world
    dist.gather_object((x, outs), gathered if rank == 0 else None, dst=0)
    ok = True
    if rank == 0:
        ref_ctx = obsmoe.MoeContext(obsmoe.MoeShape(H, I, E, K, n_layers=1, max_tokens=160), local)
        ref_ctx.load_layer(0, L)
        for r, (xr, outs_r) in enumerate(gathered):
            Tr = xr.shape[0]
            if Tr == 0:
                ok &= all(o.size == 0 for o in outs_r)
                continue
            xrd = torch.from_numpy(xr.view(np.int16)).cuda()
            rr = torch.from_numpy(O.synth_x(SEED + 1, 0, Tr, H, row0=1000 * r).view(np.int16)).cuda()
            for rep, got in enumerate(outs_r):
                ref = torch.empty((Tr, H), dtype=torch.int16, device="cuda")
                ref_ctx.moe_forward(0, xrd, ref, Tr, residual=rr if rep == 2 else None, path=obsmoe.PATH_PREFILL)
                torch.cuda.synchronize()
                want = ref.cpu().numpy().view(np.uint16)
                same = np.array_equal(got, want)
                print(f"rank {r} forward {rep}: T={Tr} bit-exact={same}", flush=True)
                ok &= same
        ref_ctx.check_device()
        ref_ctx.close()
    oks = [None] * world
    dist.all_gather_object(oks, ok_local)
    flag = [ok and all(oks)]
    dist.broadcast_object_list(flag, src=0)
    ctx.close()
    dist.destroy_process_group()
    sys.exit(0 if flag[0] else 1)


if __name__ == "__main__":
    main()
