"""One rank of the multi-GPU expert-parallel check (run by torchrun from
test_ep_multi_gpu.py, one process per GPU): config-3 shapes, this rank's
slice of the rows through an expert-parallel plan, compared bitwise with a
single-GPU plan over the same rows on the same GPU.

EP_MODE=timeout checks failure detection instead: rank 1 connects and then
never takes part in a forward (it waits, alive, at a host barrier), so rank
0's device barrier must give up after UOCR_EP_WAIT_MS and uocr_moe_check
must report UOCR_ERR_TIMEOUT — no fault, no hang."""
import datetime
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(os.path.dirname(HERE), "grpc-unlimited-ocr_b200"))


def main():
    import torch
    import torch.distributed as dist

    import ep
    import moe_configs as C
    import uocr_moe as M

    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=dev)
    strided = os.environ.get("EP_STRIDED", "0") == "1"
    balanced = os.environ.get("EP_BALANCED", "0") == "1"
    total = int(os.environ.get("EP_ROWS", "4096"))
    cfg = C.CONFIGS[3]
    start, count = ep.rows_of(total, world, rank)
    t = C.device_layer(cfg, 0, device=dev)
    owner = None
    if balanced:
        # Placement from a calibration pass: every rank's routing histogram.
        cal = M.Plan(cfg.dims(), max_rows=max(count, 17), router_bias=True, device=local)
        C.load_layer(cal, cfg, 0, t)
        xc = C.device_input(cfg, total, device=dev)[start:start + count].contiguous()
        ids = torch.empty(max(count, 1), cfg.top_k, dtype=torch.int32, device=dev)
        if count > 0:
            cal.forward(0, xc, torch.empty_like(xc), ids)
        cal.check()
        cal.close()
        mine = torch.bincount(ids[:count].reshape(-1).long(), minlength=cfg.experts)
        allc = [torch.empty_like(mine) for _ in range(world)]
        dist.all_gather(allc, mine)
        owner = ep.balanced_owner_table([c.cpu().tolist() for c in allc], world)
    plan = M.Plan(cfg.dims(), max_rows=max(count, 1), router_bias=True, device=local,
                  flags=M.PLAN_EP_STRIDED if strided else 0, ep_world=world, ep_rank=rank, ep_owner=owner)
    C.load_layer(plan, cfg, 0, t)
    ep.connect(plan)
    x = C.device_input(cfg, total, device=dev)[start:start + count].contiguous()
    y = torch.empty_like(x)
    if os.environ.get("EP_MODE") == "timeout":
        result = 0
        if rank == 0:
            plan.forward(0, x, y)
            try:
                plan.check()
                result = 1  # should not complete without the peer
            except M.UocrError as e:
                result = 0 if e.code == 6 else 2
        flag = torch.tensor([result], device=dev)
        dist.all_reduce(flag)  # rank 1 waits here, alive, until rank 0 is done
        dist.barrier()
        plan.close()
        dist.destroy_process_group()
        if rank == 0:
            print(f"EP timeout world {world}: {'EP_TIMEOUT_OK' if flag.item() == 0 else 'EP_TIMEOUT_BAD'}")
        sys.exit(0 if flag.item() == 0 else 1)
    for _ in range(3):  # repeated calls reuse the exchange buffers
        plan.forward(0, x, y)
    plan.check()
    single = M.Plan(cfg.dims(), max_rows=max(count, 17), router_bias=True, device=local)
    C.load_layer(single, cfg, 0, t)
    y1 = torch.empty_like(x)
    if count > 16:
        single.forward(0, x, y1)
        single.check()
        ok = torch.equal(y, y1)
    else:
        ok = True
    # Two layers with the residual (uocr_moe_forward_stack, captured as a CUDA
    # graph) against the same stack on one GPU.
    dims2 = cfg.dims(layers=2)
    plan2 = M.Plan(dims2, max_rows=max(count, 1), router_bias=True, device=local,
                   flags=M.PLAN_EP_STRIDED if strided else 0, ep_world=world, ep_rank=rank, ep_owner=owner)
    single2 = M.Plan(dims2, max_rows=max(count, 17), router_bias=True, device=local)
    t1 = C.device_layer(cfg, 1, device=dev)
    for pl in (plan2, single2):
        C.load_layer(pl, cfg, 0, t)
        C.load_layer(pl, cfg, 1, t1)
    ep.connect(plan2)
    s = torch.cuda.Stream(device=dev)
    h = x.clone()
    h1 = x.clone()
    with torch.cuda.stream(s):
        for _ in range(2):  # capture, then a replay
            h.copy_(x)
            plan2.forward_stack(h, stream=s)
        plan2.check(stream=s)
        if count > 16:
            single2.forward_stack(h1, stream=s)
            single2.check(stream=s)
            ok = ok and torch.equal(h, h1)
    flag = torch.tensor([0 if ok else 1], device=dev)
    dist.all_reduce(flag)
    dist.barrier()
    torch.cuda.synchronize()
    plan.close()
    single.close()
    dist.barrier()
    plan2.close()
    single2.close()
    dist.destroy_process_group()
    if rank == 0:
        print(f"EP world {world} strided {strided} balanced {balanced} rows {total}: "
              f"{'EP_OK' if flag.item() == 0 else 'EP_MISMATCH'}")
    sys.exit(0 if flag.item() == 0 else 1)


if __name__ == "__main__":
    main()
