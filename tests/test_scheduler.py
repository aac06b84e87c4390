"""Continuous-batching scheduler on CPU: same tokens as static batching, prefill interleaved with decode under a
token budget, preemption and exact resume when the KV pool runs out, idle-session eviction on deadlock."""
import torch

from arcagi2_flashnext_dots3_b200.config import EngineConfig, fn_small_config
from arcagi2_flashnext_dots3_b200.engine.llm import LLM
from arcagi2_flashnext_dots3_b200.engine.scheduler import Scheduler
from arcagi2_flashnext_dots3_b200.models import fn_weights

CFG = fn_small_config(num_layers=2, ple_layers=())
W = fn_weights.to_engine(fn_weights.random_dense(CFG, seed=0, symmetric=False), CFG, "cpu")
PROMPTS = [torch.randint(0, CFG.vocab_size, (n,), generator=torch.Generator().manual_seed(n)).tolist()
           for n in (9, 30, 17, 44, 5)]


def _llm(**kw):
    ec = dict(max_seqs=4, max_model_len=128, block_size=8, graph_batch_sizes=(1, 2, 4))
    ec.update(kw)
    return LLM(CFG, W, "cpu", EngineConfig(**ec))


def _greedy():
    llm = _llm(max_seqs=8)
    return llm.generate(PROMPTS, max_new_tokens=12)


def test_scheduler_matches_static_batching():
    want = _greedy()
    sch = Scheduler(_llm(), prefill_budget=64, chunk=16)
    assert sch.generate(PROMPTS, max_new_tokens=12) == want     # 5 requests through 4 slots
    st = sch.stats
    assert st.finished == 5 and st.generated == 60 and st.prefill_tokens == sum(map(len, PROMPTS))
    assert not sch.llm.running and len(sch.llm.free_slots) == 4 and sch.llm.alloc.n_free() == sch.llm.caches.n_blocks - 1


def test_prefill_interleaves_with_decode():
    sch = Scheduler(_llm(), prefill_budget=8, chunk=8)
    a = sch.submit(PROMPTS[0], 20)
    while not a.seq or not sch.running:
        sch.step()
    b = sch.submit(PROMPTS[3], 4)        # 44 prompt tokens: six iterations of prefill at 8 tokens each
    produced = 0
    while b.seq is None or b.seq.pos < len(PROMPTS[3]):
        out = sch.step()
        produced += len(out.get(a.rid, []))
    assert produced >= 5                  # the running sequence kept decoding during b's prefill
    sch.run()
    assert a.done and b.done


def test_preemption_and_exact_resume():
    want = _greedy()
    sch = Scheduler(_llm(kv_blocks=12), prefill_budget=64, chunk=16, watermark=0)
    got = sch.generate(PROMPTS, max_new_tokens=12)
    assert got == want
    assert sch.stats.preempted > 0


def test_idle_session_eviction_unblocks_admission():
    llm = _llm(kv_blocks=8)
    held = []
    for p in (PROMPTS[1], PROMPTS[2]):            # two idle "sessions" holding KV blocks
        s = llm.add(p, 1)
        llm.running.pop(s.slot)
        held.append(s)
    calls = []

    def evict():
        if not held:
            return False
        llm.release(held.pop())
        calls.append(1)
        return True
    sch = Scheduler(llm, evict_idle=evict, watermark=0)
    r = sch.submit(PROMPTS[3], 4)
    sch.run([r])
    assert r.done and len(calls) >= 1 and sch.stats.evicted_sessions == len(calls)


def test_sessions_keep_kv_extend_and_exact_eviction_resume():
    """A session chunk keeps its KV; a push prefills only the new tokens. An evicted idle session is rebuilt
    from its history on the next push and continues exactly as a never-evicted one."""
    def run(kv_blocks, squeeze):
        sch = Scheduler(_llm(kv_blocks=kv_blocks), prefill_budget=64, chunk=16, watermark=0)
        a = sch.submit(PROMPTS[1], 6, keep_kv=True)
        sch.run([a])
        assert a.done and a in sch.idle and a.holds_slot
        if squeeze:     # other traffic needs the blocks while `a` is idle: it gets evicted on deadlock
            sch.generate([PROMPTS[3]], max_new_tokens=30)
        sch.extend(a, [a.out[-1]] + PROMPTS[0][:5], 6)
        sch.run([a])
        pf = sch.stats.prefill_tokens
        sch.close(a)
        return list(a.seq.out), a.history, sch.stats, pf
    out_kept, hist_kept, st_kept, pf_kept = run(0, False)
    out_ev, hist_ev, st_ev, pf_ev = run(12, True)
    assert st_ev.evicted_sessions >= 1 and st_kept.evicted_sessions == 0
    assert out_ev == out_kept and hist_ev == hist_kept
    assert pf_kept == len(PROMPTS[1]) + 6        # the push prefilled only the pushed tokens


def test_idle_session_offload_to_host_tier_resumes_without_recompute():
    """With a host tier, the idle session squeezed out of the KV pool is offloaded instead of dropped: its next
    push restores blocks and recurrent state and prefills only the pushed tokens, with the same output."""
    from arcagi2_flashnext_dots3_b200.engine.kv_tier import HostKVTier

    def run(kv_blocks, squeeze, tier_blocks):
        llm = _llm(kv_blocks=kv_blocks)
        sch = Scheduler(llm, prefill_budget=64, chunk=16, watermark=0,
                        host_tier=HostKVTier(llm, tier_blocks) if tier_blocks else None)
        a = sch.submit(PROMPTS[1], 6, keep_kv=True)
        sch.run([a])
        if squeeze:
            sch.generate([PROMPTS[3]], max_new_tokens=30)
        pf0 = sch.stats.prefill_tokens
        sch.extend(a, [a.out[-1]] + PROMPTS[0][:5], 6)
        sch.run([a])
        return list(a.seq.out), sch.stats, sch.stats.prefill_tokens - pf0
    out_kept, st_kept, pf_kept = run(0, False, 0)
    out_tier, st_tier, pf_tier = run(12, True, 16)
    assert st_tier.offloaded_sessions >= 1 and st_tier.restored_sessions >= 1 and st_tier.evicted_sessions == 0
    assert out_tier == out_kept
    assert pf_tier == pf_kept == 6            # the push only: no recompute of the context
