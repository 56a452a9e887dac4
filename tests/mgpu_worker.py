"""One rank of the multi-GPU parity check (launched by tests/test_gpu_multigpu.py under torchrun).

Llama-3-70B decode shapes: Q4_K_M 8192 -> 28672 and 28672 -> 8192, Q6_K
lm_head 8192 -> 128256, plus a Q8_0 prefill GEMM (512 tokens, 8192 -> 28672). Every rank
uploads only its output-row shard (jkb200.shard.shard_rows), computes it with the same kernels
as a single-GPU call, and one NCCL all-gather collects the slices. Rank 0 also holds the full
matrices and checks that the reassembled outputs equal the single-GPU results bit for bit: rows
are independent, so sharding by rows changes no arithmetic (gemv_repacked_rows, repack.rs:4014).
The same shapes then go through the library's one-kernel all-gather (jkb200.shard.PeerOutputs:
every rank pushes its rows into every peer's buffer over NVLink): over three steps alternating
the two output slots, every rank's full outputs must equal its own single-GPU results bit for
bit. Then the same with pushed outputs (the GEMV kernels store each row into every peer's
buffer, one signal kernel a step): single, grouped f32-input and token-batch launches. Prints
one JSON line per rank and exits non-zero on a mismatch.
"""
import json
import os
import sys
from datetime import timedelta

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "jero-kernels-rvv_b200"))
sys.path.insert(0, ROOT)

import bench  # noqa: E402  (seeded synthetic GGUF matrices)
import jkb200 as jkb  # noqa: E402
from jkb200.shard import PeerOutputs, ShardedOutputs, shard_rows  # noqa: E402

Q4_K, Q6_K, Q8_0 = 12, 14, 8
MATS = [("ffn_gate", Q4_K, 28672, 8192, "h"), ("ffn_down", Q4_K, 8192, 28672, "a"),
        ("lm_head", Q6_K, 128256, 8192, "f")]
ACTS = {"h": 8192, "a": 28672, "f": 8192}


def main():
    world = int(os.environ["WORLD_SIZE"])
    rank = int(os.environ["RANK"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", local))
    g = torch.Generator().manual_seed(11)
    xs = {s: torch.randn(n, generator=g).cuda() for s, n in ACTS.items()}
    xq = {s: jkb.empty_q8_k_blocks(n // 256) for s, n in ACTS.items()}
    for s in ACTS:
        jkb.quantize_row_q8_k(xs[s], xq[s])
    outs = ShardedOutputs([(n, r) for n, _, r, _, _ in MATS], world, rank)
    full_raw = {}
    for i, (name, quant, rows, cols, s) in enumerate(MATS):
        rr = outs.rows_of(name)
        raw = bench.synth_matrix(quant, rows, cols, 500 + i, rr.start, rr.stop)
        w = jkb.Weight(jkb.TensorView(name, quant, [len(rr), cols], raw), len(rr), cols)
        fn = jkb.gemv_q4_k_q8_k if quant == Q4_K else jkb.gemv_q6_k_q8_k
        fn(outs.local_slice(name), w, xq[s])
        if rank == 0:
            full_raw[name] = bench.synth_matrix(quant, rows, cols, 500 + i)
    outs.gather()

    # prefill GEMM, weight rows sharded the same way; its output is [m][rows], so each rank
    # sends its slice transposed ([rows][m]) and rank 0 transposes the concatenation back
    m, n, k = 512, 28672, 8192
    rr = shard_rows(n, world, rank)
    raw = bench.synth_matrix(Q8_0, n, k, 600, rr.start, rr.stop)
    rw = jkb.RepackedWeight.from_tensor(jkb.TensorView("w", Q8_0, [len(rr), k], raw), len(rr), k)
    x = torch.randn(m * k, generator=torch.Generator().manual_seed(12)).cuda()
    act = jkb.QuantizedActQ8.quantize(x, m, k)
    part = torch.empty(m * len(rr), dtype=torch.float32, device="cuda")
    rw.gemm(part, act)
    slab = part.view(m, len(rr)).t().contiguous().view(-1)
    gathered = [torch.empty(m * len(shard_rows(n, world, r)), dtype=torch.float32, device="cuda")
                for r in range(world)]
    dist.all_gather(gathered, slab)
    torch.cuda.synchronize()

    res = {"rank": rank, "world": world}
    ok = True
    if rank == 0:
        for i, (name, quant, rows, cols, s) in enumerate(MATS):
            w = jkb.Weight(jkb.TensorView(name, quant, [rows, cols], full_raw[name]), rows, cols)
            ref = torch.empty(rows, dtype=torch.float32, device="cuda")
            fn = jkb.gemv_q4_k_q8_k if quant == Q4_K else jkb.gemv_q6_k_q8_k
            fn(ref, w, xq[s])
            same = torch.equal(outs.output(name).view(torch.int32), ref.view(torch.int32))
            res[name] = "bit-exact" if same else "MISMATCH"
            ok &= same
        rwf = jkb.RepackedWeight.from_tensor(
            jkb.TensorView("w", Q8_0, [n, k], bench.synth_matrix(Q8_0, n, k, 600)), n, k)
        ref = torch.empty(m * n, dtype=torch.float32, device="cuda")
        rwf.gemm(ref, act)
        got = torch.cat(gathered).view(n, m).t().contiguous().view(-1)
        same = torch.equal(got.view(torch.int32), ref.view(torch.int32))
        res["prefill_gemm"] = "bit-exact" if same else "MISMATCH"
        ok &= same
        res["device_status"] = jkb.device_status()
    # the library's one-kernel all-gather over NVLink: every rank computes its rows into their
    # global positions and pushes them to every peer; three steps alternate the two slots with
    # fresh inputs, and after each every rank checks all rows against its own single-GPU
    # computation of the full matrices
    torch.cuda.synchronize()
    dist.barrier()
    pouts = PeerOutputs([(nm, r) for nm, _, r, _, _ in MATS], world, rank)
    shard_w, full_w = {}, {}
    for i, (name, quant, rows, cols, s) in enumerate(MATS):
        rr = pouts.rows_of(name)
        raw = bench.synth_matrix(quant, rows, cols, 700 + i)
        row_bytes = raw.size // rows
        shard_w[name] = jkb.Weight(jkb.TensorView(name, quant, [len(rr), cols],
                                                  raw[rr.start * row_bytes:rr.stop * row_bytes]),
                                   len(rr), cols)
        full_w[name] = jkb.Weight(jkb.TensorView(name, quant, [rows, cols], raw), rows, cols)
    peer_ok = True
    for step in range(3):
        slot = step % 2
        gs = torch.Generator().manual_seed(100 + step)
        xq_s = {}
        for s_, n_ in ACTS.items():
            xq_s[s_] = jkb.empty_q8_k_blocks(n_ // 256)
            jkb.quantize_row_q8_k(torch.randn(n_, generator=gs).cuda(), xq_s[s_])
        for name, quant, rows, cols, s in MATS:
            jkb.gemv_rows(pouts.local_slice(name, slot), shard_w[name], xq_s[s],
                          range(0, len(pouts.rows_of(name))))
        pouts.gather(slot)
        for name, quant, rows, cols, s in MATS:
            ref = torch.empty(rows, dtype=torch.float32, device="cuda")
            jkb.gemv_rows(ref, full_w[name], xq_s[s], range(0, rows))
            peer_ok &= torch.equal(pouts.output(name, slot).view(torch.int32),
                                   ref.view(torch.int32))
        torch.cuda.synchronize()
    res["peer_allgather"] = "bit-exact" if peer_ok else "MISMATCH"
    res["peer_status"] = jkb.device_status()
    ok &= peer_ok and res["peer_status"] == 0
    torch.cuda.synchronize()
    dist.barrier()  # no rank still writes into a peer's buffer
    pouts.destroy()

    # pushed outputs: the GEMVs store their rows into every peer's buffer as they compute them
    # and one signal kernel a step completes the exchange. ffn_gate through the grouped
    # f32-input launch, ffn_down and lm_head through pre-quantized gemv_rows; then a batch of
    # four tokens through gemv_batch. Every rank checks every row.
    push = PeerOutputs([(nm, r) for nm, _, r, _, _ in MATS], world, rank, push=True)
    push_ok = True
    for step in range(3):
        slot = step % 2
        gs = torch.Generator().manual_seed(200 + step)
        x_s = {s_: torch.randn(n_, generator=gs).cuda() for s_, n_ in ACTS.items()}
        xq_s = {}
        for s_, n_ in ACTS.items():
            xq_s[s_] = jkb.empty_q8_k_blocks(n_ // 256)
            jkb.quantize_row_q8_k(x_s[s_], xq_s[s_])
        for name, quant, rows, cols, s in MATS:
            if name == "ffn_gate":
                jkb.vec_dot_grouped_rvv([(push.local_slice(name, slot), shard_w[name])], x_s[s])
            else:
                jkb.gemv_rows(push.local_slice(name, slot), shard_w[name], xq_s[s],
                              range(0, len(push.rows_of(name))))
        push.gather(slot)
        for name, quant, rows, cols, s in MATS:
            ref = torch.empty(rows, dtype=torch.float32, device="cuda")
            if name == "ffn_gate":
                jkb.vec_dot_grouped_rvv([(ref, full_w[name])], x_s[s])
            else:
                jkb.gemv_rows(ref, full_w[name], xq_s[s], range(0, rows))
            push_ok &= torch.equal(push.output(name, slot).view(torch.int32),
                                   ref.view(torch.int32))
        torch.cuda.synchronize()
    torch.cuda.synchronize()
    dist.barrier()
    push.destroy()
    name, quant, rows, cols, s = MATS[2]
    pb = PeerOutputs([(name, rows)], world, rank, batch=4, push=True)
    xb = torch.randn(4 * cols, generator=torch.Generator().manual_seed(300)).cuda()
    xqb = jkb.empty_q8_k_blocks(4 * cols // 256)
    jkb.quantize_rows_q8_k(xb, 4, cols, xqb)
    jkb.gemv_batch(pb.local_slice(name, 0), shard_w[name], xqb, 4)
    pb.gather(0)
    ref = torch.empty(4 * rows, dtype=torch.float32, device="cuda")
    jkb.gemv_batch(ref, full_w[name], xqb, 4)
    push_ok &= torch.equal(pb.output(name, 0).reshape(-1).view(torch.int32),
                           ref.view(torch.int32))
    res["peer_push"] = "bit-exact" if push_ok else "MISMATCH"
    res["push_status"] = jkb.device_status()
    ok &= push_ok and res["push_status"] == 0
    torch.cuda.synchronize()
    dist.barrier()
    pb.destroy()

    res["ok"] = bool(ok)
    print(json.dumps(res), flush=True)
    dist.barrier()
    dist.destroy_process_group()
    sys.exit(0 if ok else 1)


if __name__ == "__main__":
    main()
