"""A scripted scheduler session, run once against the reference's
``scheduler/continuous_batch.py`` (by ``make_golden.py``, fixture
``scheduler_trace.npz``) and again against ``hydranet_b200.batching`` by
``tests/test_batching_cpu.py``: the two traces must be equal line for line.

``mod`` is the module under test; it must provide ``Request``,
``RequestState``, ``ContinuousBatcher``, ``MicrobatchScheduler`` and
``PrefetchSchedule`` with the reference's interface.  Nothing timing-dependent
is recorded (only whether a timestamp was set)."""


def run(mod, torch):
    lines = []
    b = mod.ContinuousBatcher(max_batch_size=3, max_queue_size=4)
    reqs = [mod.Request(f"r{i}", torch.arange(3 + i), max_tokens=2 + i) for i in range(7)]

    def show(bt):
        if bt is None:
            lines.append("batch None")
            return
        lines.append(f"batch {bt.batch_id} size {bt.batch_size} prefill {bt.is_prefill} "
                     + " ".join(f"{r.request_id}:{r.state.value}" for r in bt.requests))

    def stats():
        lines.append("stats " + " ".join(f"{k}={v}" for k, v in sorted(b.get_stats().items())))

    for r in reqs[:5]:
        lines.append(f"submit {r.request_id} {b.submit(r)} {r.state.value}")
    stats()
    show(b.get_batch(timeout_ms=1))
    stats()
    reqs[1].state = mod.RequestState.GENERATING
    reqs[0].state = mod.RequestState.GENERATING
    show(b.get_batch(timeout_ms=1))
    b.complete_request("r1")
    lines.append(f"r1 {reqs[1].state.value} end {reqs[1].end_time is not None} start {reqs[1].start_time is not None}")
    show(b.get_batch(timeout_ms=1))
    b.cancel_request("r0")
    lines.append(f"r0 {reqs[0].state.value} end {reqs[0].end_time is not None}")
    b.complete_request("missing")
    b.cancel_request("r0")
    stats()
    lines.append(f"submit r5 {b.submit(reqs[5])}")
    lines.append(f"submit r6 {b.submit(reqs[6])}")
    show(b.get_batch(timeout_ms=1))
    # an active request that is no longer active (state changed outside) is skipped
    reqs[2].state = mod.RequestState.COMPLETED
    show(b.get_batch(timeout_ms=1))
    stats()
    for rid in sorted(b.active_requests):
        b.complete_request(rid)
    show(b.get_batch(timeout_ms=1))
    for rid in sorted(b.active_requests):
        b.complete_request(rid)
    show(b.get_batch(timeout_ms=1))
    stats()
    lines.append("completed " + " ".join(f"{k}:{v.state.value}" for k, v in sorted(b.completed_requests.items())))
    r = reqs[3]
    r.generated_ids.extend([5, 6])
    lines.append(f"r3 total {r.total_tokens} active {r.is_active}")
    lines.append(f"next_batch_id {b.next_batch_id}")

    ms = mod.MicrobatchScheduler(microbatch_size=4)
    for mb, s in ms.split_prefill(torch.arange(10).view(1, 10)):
        lines.append(f"mb {s} {mb.tolist()}")
    for mb, s in mod.MicrobatchScheduler(microbatch_size=5).split_prefill(torch.arange(10).view(1, 10)):
        lines.append(f"mb5 {s} {mb.shape[1]}")
    lines.append(f"prefetch {ms.get_prefetch_experts([(0, 1), (0, 3)], 1, 3)} {ms.get_prefetch_experts([(0, 1)], 3, 3)}")
    ps = mod.PrefetchSchedule(num_layers=2, num_experts=8, num_streams=2)
    lines.append(f"ps {ps.schedule_prefetch(0, [1], [2, 3, 2])}")
    lines.append(f"ps {ps.schedule_prefetch(0, [1], [3, 4, 5])}")
    lines.append(f"ps {ps.schedule_prefetch(1, [1], None)}")
    lines.append(f"ps {ps.schedule_prefetch(1, [1], [3])}")
    ps.clear()
    lines.append(f"ps {ps.schedule_prefetch(0, [1], [2])}")
    return lines
