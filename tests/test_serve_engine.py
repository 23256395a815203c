"""The serving engine and its OpenAI front on CPU (deterministic stand-in
model): continuous batching admits new requests between decode steps and
keeps every request's KV consistent, KV reservations bound admission and are
returned on finish / cancel / error, a failed step fails only its requests,
the HTTP routes answer like the engine API the proxy drives, and the retry /
resume proxy in front of two engines turns a failed stream into the
uninterrupted output."""
import asyncio
import threading
import time

import aiohttp
import pytest

from connex.serving.fake_backend import reference
from connex_b200.serve.api import Server, WordCodec
from connex_b200.serve.engine import EngineFull, GenerationEngine, RuleStepper
from connex_b200.serve.pipeline import split_layers
from tests.helpers import wait_until
from tests.test_serving import _proxy, _run, _serve, _stream, _text


def _collect(engine, prompt, n, **kw):
    done = threading.Event()
    out = {"toks": [], "reason": None}

    def cb(r, tok, reason):
        if tok is not None:
            out["toks"].append(tok)
        if reason:
            out["reason"] = reason
            done.set()
    out["req"] = engine.submit(prompt, n, cb, **kw)
    out["done"] = done
    return out


def test_batching_matches_the_uninterrupted_rule_and_admits_between_steps():
    st = RuleStepper(step_delay_s=0.002)
    eng = GenerationEngine(st, chunked=False).start()        # separate prefill and decode steps
    try:
        a = _collect(eng, [1, 5, 6], 60)
        assert wait_until(lambda: len(a["toks"]) >= 2, 5)
        b = _collect(eng, [1, 7], 8)                    # joins while a is decoding
        for x in (a, b):
            assert x["done"].wait(5)
        assert a["toks"] == reference([1, 5, 6], 60)[0] and a["reason"] == "length"
        assert b["toks"] == reference([1, 7], 8)[0]
        kinds = [k for k, _ in st.calls]
        assert kinds.count("prefill") == 2
        mixed = [rids for k, rids in st.calls if k == "decode" and len(rids) == 2]
        assert mixed                                    # a and b decoded in the same step
        assert wait_until(lambda: not st.held and eng.blocks_reserved == 0, 5)
    finally:
        eng.stop()


def test_chunked_prefill_reads_long_prompts_while_others_decode():
    st = RuleStepper(step_delay_s=0.001)
    eng = GenerationEngine(st, max_step_tokens=64).start()
    try:
        a = _collect(eng, [1, 5, 6], 40)
        assert wait_until(lambda: len(a["toks"]) >= 2, 5)
        long = [1] + [(7 * i) % 900 + 3 for i in range(299)]  # 300 tokens: five chunks of <= 64
        b = _collect(eng, long, 6)
        for x in (a, b):
            assert x["done"].wait(10)
        assert a["toks"] == reference([1, 5, 6], 40)[0]
        assert b["toks"] == reference(long, 6)[0]                 # the same as one whole prefill
        steps = [(k, rids) for k, rids in st.calls]
        with_b = [i for i, (k, rids) in enumerate(steps) if b["req"].rid in rids]
        chunk_steps = with_b[:5]
        assert all(steps[i][0] == "mixed" and a["req"].rid in steps[i][1] for i in chunk_steps[:4])
        assert eng.stats["chunks"] >= 5 and b["req"].t_first is not None
        # a kept decoding: one token per step while b's prompt was read
        assert all(a["req"].rid in steps[i][1] for i in chunk_steps[:4])
        assert wait_until(lambda: not st.held and eng.blocks_reserved == 0, 5)
        # the budget is shared: two long prompts never exceed it in one step
        st.calls.clear()
        c, d = _collect(eng, long, 3), _collect(eng, long[::-1], 3)
        for x in (c, d):
            assert x["done"].wait(10)
        assert c["toks"] == reference(long, 3)[0] and d["toks"] == reference(long[::-1], 3)[0]
    finally:
        eng.stop()


def test_chunked_steps_never_exceed_the_budget():
    seen = []

    class Spy(RuleStepper):
        def mixed(self, rids, seqs, ctx, n_new):
            seen.append(sum(n_new))
            return super().mixed(rids, seqs, ctx, n_new)
    st = Spy(step_delay_s=0.0005)
    eng = GenerationEngine(st, max_step_tokens=50).start()
    try:
        outs = [_collect(eng, [1] + [3 + k % 7] * (30 + 17 * k), 5) for k in range(6)]
        for o in outs:
            assert o["done"].wait(10)
        assert max(seen) <= 50 and len(seen) > 6
    finally:
        eng.stop()


def test_stop_ids_cancel_and_kv_reservations():
    st = RuleStepper(num_blocks=4, step_delay_s=0.002)        # 4 blocks of 16 tokens
    eng = GenerationEngine(st).start()
    try:
        stop_at = reference([1, 5], 6)[0][2]
        s = _collect(eng, [1, 5], 6, stop_ids=[stop_at])
        assert s["done"].wait(5) and s["reason"] == "stop" and s["toks"][-1] == stop_at and len(s["toks"]) == 3
        big = _collect(eng, [1] * 10, 40)                     # 50 tokens: 4 blocks, the whole cache
        assert wait_until(lambda: len(big["toks"]) >= 1, 5)
        small = _collect(eng, [1, 2], 3)                      # waits for the blocks
        time.sleep(0.05)
        assert small["toks"] == [] and eng.load()["waiting"] == 1
        eng.cancel(big["req"])
        assert big["done"].wait(5) and big["reason"] == "abort"
        assert small["done"].wait(5) and small["toks"] == reference([1, 2], 3)[0]
        with pytest.raises(EngineFull):
            eng.submit([1] * 10, 60, lambda *a: None)         # 70 tokens > 4 blocks
        with pytest.raises(EngineFull):
            eng.submit([1] * 4000, 200, lambda *a: None)      # beyond the context
        with pytest.raises(ValueError):
            eng.submit([1, 5000], 2, lambda *a: None)         # outside the vocabulary
        assert wait_until(lambda: eng.blocks_reserved == 0 and not st.held, 5)   # released right after the callback
    finally:
        eng.stop()


def test_a_failed_step_fails_only_its_requests():
    boom = {"on": False}
    st = RuleStepper(step_delay_s=0.002, fail_on=lambda kind, rids: boom["on"] and kind == "decode")
    eng = GenerationEngine(st).start()
    try:
        a = _collect(eng, [1, 3], 50)
        time.sleep(0.02)
        boom["on"] = True
        assert a["done"].wait(5) and a["reason"] == "error" and a["req"].error.startswith("RuntimeError")
        boom["on"] = False
        b = _collect(eng, [1, 4], 5)
        assert b["done"].wait(5) and b["toks"] == reference([1, 4], 5)[0]
        assert wait_until(lambda: eng.alive and eng.stats["step_errors"] == 1 and not st.held, 5)
    finally:
        eng.stop()


def test_http_routes():
    async def main():
        eng = GenerationEngine(RuleStepper(step_delay_s=0.001)).start()
        srv = Server(eng, "m")
        runner, url = await _serve(srv.app())
        try:
            async with aiohttp.ClientSession() as s:
                assert (await (await s.get(url + "/health")).json())["status"] == "ok"
                assert (await (await s.get(url + "/v1/models")).json())["data"][0]["id"] == "m"
                r = await (await s.post(url + "/v1/completions", json={"prompt": "t5 t6", "max_tokens": 4,
                                                                       "return_token_ids": True})).json()
                ids, text = reference("t5 t6", 4)
                assert r["choices"][0]["text"] == text and r["choices"][0]["token_ids"] == ids
                assert r["usage"] == {"prompt_tokens": 3, "completion_tokens": 4, "total_tokens": 7}
                tok = await (await s.post(url + "/tokenize", json={"prompt": "t5 t6"})).json()
                assert tok["tokens"] == [1, 5, 6]
                det = await (await s.post(url + "/detokenize", json={"tokens": [5, 6]})).json()
                assert det["prompt"] == " t5 t6"
                bad = await s.post(url + "/v1/completions", json={"prompt": "t1", "max_tokens": 5000})
                assert bad.status == 400
                bad = await s.post(url + "/v1/completions", json={"prompt": "t1", "n": 2})
                assert bad.status == 400
                load = await (await s.get(url + "/load")).json()
                assert load["running"] == 0 and load["tokens"] == 4
                m = await (await s.get(url + "/metrics")).text()
                assert 'connex_serve_requests_total{finish_reason="length"} 1.0' in m
                assert "connex_serve_generated_tokens_total 4.0" in m and "connex_serve_ttft_seconds_count 1.0" in m
                assert "connex_serve_waiting 0.0" in m
            chunks, done = await _stream(url, "/v1/completions",
                                         {"prompt": [1, 9, 9], "max_tokens": 5, "return_token_ids": True,
                                          "logprobs": 0, "return_tokens_as_token_ids": True,
                                          "stream_options": {"include_usage": True, "continuous_usage_stats": True}})
            assert done and _text(chunks) == reference([1, 9, 9], 5)[1]
            toks = [c["choices"][0]["token_ids"][0] for c in chunks if c["choices"]]
            assert toks == reference([1, 9, 9], 5)[0]
            lp = chunks[0]["choices"][0]["logprobs"]
            assert lp["tokens"] == [f"token_id:{toks[0]}"] and lp["token_logprobs"] == [None]
            assert chunks[-1]["usage"]["completion_tokens"] == 5 and chunks[-1]["choices"] == []
            assert chunks[-2]["choices"][0]["finish_reason"] == "length"
            msgs = [{"role": "user", "content": "t7 t8"}]
            chunks, done = await _stream(url, "/v1/chat/completions", {"messages": msgs, "max_tokens": 3})
            ids = WordCodec(1000).chat(msgs)
            assert done and _text(chunks, chat=True) == reference(ids, 3)[1]
        finally:
            await runner.cleanup()
            eng.stop()
    _run(main())


def test_resume_proxy_turns_a_failed_engine_stream_into_the_full_output():
    async def main():
        trip = {"n": 0}

        def fail_once(kind, rids):              # engine A fails its 4th decode step, once
            if kind == "decode":
                trip["n"] += 1
                return trip["n"] == 4
            return False
        ea = GenerationEngine(RuleStepper(step_delay_s=0.002, fail_on=fail_once)).start()
        eb = GenerationEngine(RuleStepper(step_delay_s=0.002)).start()
        ra, ua = await _serve(Server(ea, "m").app())
        rb, ub = await _serve(Server(eb, "m").app())
        p = _proxy([ua, ub])
        pr, url = await _serve(p.app())
        try:
            for _ in range(2):                  # whichever replica the proxy picks first
                chunks, done = await _stream(url, "/v1/completions", {"model": "m", "prompt": "t3 t4",
                                                                      "max_tokens": 12})
                assert done and _text(chunks) == reference("t3 t4", 12)[1]
            assert trip["n"] >= 4 and p.stats["resumes"] >= 1
        finally:
            for r in (pr, ra, rb):
                await r.cleanup()
            ea.stop()
            eb.stop()
    _run(main())


def test_split_layers():
    assert split_layers(32, 2) == [(0, 16), (16, 32)]
    assert split_layers(32, 3, "10,20") == [(0, 10), (10, 20), (20, 32)]
    for bad in ((32, 2, "40"), (32, 3, "20,10"), (32, 2, "4,8")):
        with pytest.raises(ValueError):
            split_layers(*bad)


def test_server_cli_serves_the_rule_model(tmp_path):
    """``python -m connex_b200.serve --rule`` starts, answers /health and a
    completion with the uninterrupted rule output, and exits on SIGTERM."""
    import json as _json
    import os
    import signal
    import subprocess
    import sys
    import urllib.request

    from tests.helpers import free_port, wait_until
    port = free_port()
    env = dict(os.environ, PYTHONPATH=os.getcwd())
    p = subprocess.Popen([sys.executable, "-m", "connex_b200.serve", "--rule", "--port", str(port), "--host",
                          "127.0.0.1", "--max-ctx", "512"], env=env, stdout=subprocess.PIPE,
                         stderr=subprocess.STDOUT)
    url = f"http://127.0.0.1:{port}"

    def up():
        try:
            return urllib.request.urlopen(url + "/health", timeout=1).status == 200
        except OSError:
            return False
    try:
        assert wait_until(up, 60), p.stdout.read1(4096) if p.poll() is not None else "no /health"
        req = urllib.request.Request(url + "/v1/completions", data=_json.dumps(
            {"prompt": "t5 t6", "max_tokens": 6}).encode(), headers={"Content-Type": "application/json"})
        body = _json.loads(urllib.request.urlopen(req, timeout=10).read())
        assert body["choices"][0]["text"] == reference("t5 t6", 6)[1]
    finally:
        p.send_signal(signal.SIGTERM)
        try:
            assert p.wait(20) == 0
        finally:
            if p.poll() is None:
                p.kill()


def _tp_rank(rank, port, q):
    import os
    import torch.distributed as dist
    from connex_b200.serve.engine import GenerationEngine, TPStepper, tp_follow
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=2)
        inner = RuleStepper(step_delay_s=0.001)
        if rank == 0:
            eng = GenerationEngine(TPStepper(inner)).start()
            outs = [_collect(eng, [1, 5, 6], 12), _collect(eng, [1, 7], 5)]
            for o in outs:
                assert o["done"].wait(10)
            eng.stop()
            eng.s.close()
            q.put((0, inner.calls, [o["toks"] for o in outs], dict(inner.held)))
        else:
            n = tp_follow(inner)
            q.put((1, inner.calls, n, dict(inner.held)))
        dist.destroy_process_group()
    except Exception as e:  # noqa: BLE001
        q.put((rank, "error", repr(e), None))


def test_tensor_parallel_ranks_follow_rank_zero_step_for_step():
    import torch.multiprocessing as mp
    from tests.helpers import free_port
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    ps = [ctx.Process(target=_tp_rank, args=(r, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = {r[0]: r[1:] for r in (q.get(timeout=120) for _ in range(2))}
    for p in ps:
        p.join(30)
    assert res[0][0] != "error" and res[1][0] != "error", res
    calls0, toks, held0 = res[0]
    calls1, n, held1 = res[1]
    assert calls0 == calls1 and n == len(calls0)             # the same steps, same order, same rows
    assert toks == [reference([1, 5, 6], 12)[0], reference([1, 7], 5)[0]]
    assert held0 == held1 == {}                              # releases followed too


def _tp_rank_failing(rank, port, q, failing_rank):
    """Rank ``failing_rank``'s inner stepper raises on its 3rd decode step."""
    import os
    from datetime import timedelta
    import torch.distributed as dist
    from connex_b200.serve.engine import EngineFull, GenerationEngine, GroupStepError, TPStepper, tp_follow
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=2, timeout=timedelta(seconds=10))
        seen = {"decode": 0}

        def fail_on(kind, rids):
            seen[kind] = seen.get(kind, 0) + 1
            return rank == failing_rank and kind == "decode" and seen["decode"] == 3
        inner = RuleStepper(step_delay_s=0.001, fail_on=fail_on)
        if rank == 0:
            stepper = TPStepper(inner)
            eng = GenerationEngine(stepper).start()
            out = _collect(eng, [1, 5, 6], 12)
            assert out["done"].wait(30)
            assert wait_until(lambda: not eng.alive, 30)
            try:
                eng.submit([1, 2], 3, lambda *a: None)
                refused = False
            except EngineFull:
                refused = True
            q.put((0, eng.error, out["reason"], len(out["toks"]), refused))
            eng.stop()
            stepper.close()        # as the server does at shutdown: the abort notice goes out first
        else:
            try:
                tp_follow(inner)
                q.put((1, "returned", None, None, None))
            except GroupStepError as e:
                q.put((1, "GroupStepError", str(e), None, None))
            except Exception as e:  # noqa: BLE001 - its own injected failure
                q.put((1, type(e).__name__, str(e), None, None))
                q.close()
                q.join_thread()        # the result is flushed; now die like a crashed rank
                os._exit(0)
        try:
            dist.destroy_process_group()
        except Exception:  # noqa: BLE001
            pass
    except Exception as e:  # noqa: BLE001
        q.put((rank, "error", repr(e), None, None))


def _run_tp_failing(failing_rank):
    import torch.multiprocessing as mp
    from tests.helpers import free_port
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    ps = [ctx.Process(target=_tp_rank_failing, args=(r, port, q, failing_rank)) for r in range(2)]
    for p in ps:
        p.start()
    res = {r[0]: r[1:] for r in (q.get(timeout=120) for _ in range(2))}
    for p in ps:
        p.join(30)
        if p.is_alive():
            p.kill()
    return res


def test_tensor_parallel_step_failure_on_rank_zero_stops_the_whole_group():
    res = _run_tp_failing(0)
    err, reason, n_toks, refused = res[0]
    assert err is not None and "GroupStepError" in err, res    # fatal, not a per-request failure
    assert reason == "abort" and n_toks < 12 and refused
    assert res[1][0] == "GroupStepError" and "injected decode failure" in res[1][1]   # the follower was told


def test_tensor_parallel_step_failure_on_a_follower_stops_rank_zero():
    res = _run_tp_failing(1)
    assert res[1][0] == "RuntimeError"                          # the follower's own step failed; it exited
    err, reason, n_toks, refused = res[0]
    assert err is not None and "GroupStepError" in err, res    # rank 0's next collective failed: fatal
    assert reason == "abort" and n_toks < 12 and refused


def test_stop_strings_end_generation_and_are_not_shown():
    from connex_b200.serve.api import StopMatcher
    m = StopMatcher(["END", "xyz"])
    assert m.feed("abc E") == ("abc ", False)              # "E" may start "END": held back
    assert m.feed("N") == ("", False)
    assert m.feed("Dmore") == ("", True)                    # stop completed; nothing after it shown
    m = StopMatcher("xyz")
    assert m.feed("ab x") == ("ab ", False) and m.flush() == "x"

    async def main():
        eng = GenerationEngine(RuleStepper(step_delay_s=0.001)).start()
        runner, url = await _serve(Server(eng, "m").app())
        try:
            ids, _ = reference("t5 t6", 12)
            stop = f" t{ids[3]} t{ids[4]}"                     # spans two tokens
            want = "".join(f" t{t}" for t in ids[:3])
            async with aiohttp.ClientSession() as s:
                r = await (await s.post(url + "/v1/completions", json={"prompt": "t5 t6", "max_tokens": 12,
                                                                       "stop": stop})).json()
            assert r["choices"][0]["text"] == want and r["choices"][0]["finish_reason"] == "stop"
            chunks, done = await _stream(url, "/v1/completions", {"prompt": "t5 t6", "max_tokens": 12,
                                                                   "stop": [stop]})
            assert done and _text(chunks) == want
            assert chunks[-1]["choices"][0]["finish_reason"] == "stop"
            for _ in range(100):
                if eng.stats["finished_abort"] >= 2 and eng.blocks_reserved == 0:
                    break
                await asyncio.sleep(0.05)
            assert eng.stats["finished_abort"] >= 2 and eng.blocks_reserved == 0     # generation was cut short
        finally:
            await runner.cleanup()
            eng.stop()
    _run(main())


def test_agent_sessions_stick_migrate_and_fail_over_across_engines():
    """The session proxy in front of two engines: turns stick to one engine,
    a migration re-prefills the conversation on the other (a 1-token chat
    continuation), and when the placement dies the next turn fails over."""
    from connex.agents import SessionProxy
    from connex.serving.proxy import Pool

    async def main():
        engines = [GenerationEngine(RuleStepper(step_delay_s=0.001)).start() for _ in range(2)]
        served = [await _serve(Server(e, "m").app()) for e in engines]
        urls = [u for _, u in served]
        sp = SessionProxy(Pool(urls), probe_interval=0, idle_timeout=0.5)
        pr, url = await _serve(sp.app())
        try:
            msgs = [{"role": "user", "content": "t1 t2"}]
            outs = []
            for _ in range(2):
                chunks, done = await _stream(url, "/v1/chat/completions",
                                             {"messages": msgs, "max_tokens": 3, "session_id": "s1"})
                assert done
                outs.append(_text(chunks, chat=True))
            assert outs[0] == outs[1] == reference(WordCodec(1000).chat(msgs), 3)[1]
            first = urls.index(sp.sessions["s1"].url)
            assert engines[first].stats["submitted"] == 2 and engines[1 - first].stats["submitted"] == 0
            rec = await sp.migrate("s1", urls[1 - first])
            assert rec["mode"] == "reprefill" and sp.sessions["s1"].url == urls[1 - first]
            assert engines[1 - first].stats["submitted"] == 1                   # the re-prefill
            await served[1 - first][0].cleanup()                                 # the new placement dies
            engines[1 - first].stop()
            chunks, done = await _stream(url, "/v1/chat/completions", {"messages": msgs, "max_tokens": 3},
                                         headers={"X-Connex-Session": "s1"})
            assert done and sp.stats["failovers"] == 1 and sp.sessions["s1"].url == urls[first]
        finally:
            await pr.cleanup()
            await served[first][0].cleanup()
            for e in engines:
                e.stop()
    _run(main())


def _tiny_bpe_dir(tmp_path):
    """A byte-level BPE tokenizer trained here on a few lines (no network),
    saved as an HF tokenizer directory with an EOS special token."""
    from tokenizers import Tokenizer, decoders, models, pre_tokenizers, trainers
    from transformers import PreTrainedTokenizerFast
    tk = Tokenizer(models.BPE())
    tk.pre_tokenizer = pre_tokenizers.ByteLevel(add_prefix_space=False)
    tk.decoder = decoders.ByteLevel()
    trainer = trainers.BpeTrainer(vocab_size=300, special_tokens=["<|bos|>", "<|eot|>"],
                                  initial_alphabet=pre_tokenizers.ByteLevel.alphabet())
    tk.train_from_iterator(["hello world", "the cat sat", "ok ok ok"], trainer)
    fast = PreTrainedTokenizerFast(tokenizer_object=tk, bos_token="<|bos|>", eos_token="<|eot|>")
    fast.chat_template = ("{% for m in messages %}{{ m['role'] }}: {{ m['content'] }}<|eot|>{% endfor %}"
                          "{% if add_generation_prompt %}assistant: {% endif %}")
    fast.save_pretrained(str(tmp_path))
    return str(tmp_path)


class _ScriptStepper(RuleStepper):
    """Emits a fixed continuation, whatever the prompt."""

    def __init__(self, script):
        super().__init__(vocab_size=100000)
        self.script = list(script)
        self.pos = {}

    def _step(self, kind, rids, seqs):
        out = []
        for r, s in zip(rids, seqs):
            i = self.pos.get(r, 0)
            self.pos[r] = i + 1
            self.held[r] = len(s)
            out.append(self.script[min(i, len(self.script) - 1)])
        return out


def test_streamed_text_keeps_multibyte_characters_whole_and_drops_eos(tmp_path):
    from connex_b200.serve.api import HFCodec
    codec = HFCodec(_tiny_bpe_dir(tmp_path))
    want = "héllo ✓ wörld ok"
    ids = codec.encode(want, add_special=False)
    # the characters outside the training text are split over several byte ids
    assert any("�" in codec.tok.decode([t]) for t in ids)
    script = ids + [codec.eos_id]

    async def main():
        eng = GenerationEngine(_ScriptStepper(script)).start()
        runner, url = await _serve(Server(eng, "m", codec=codec).app())
        try:
            async with aiohttp.ClientSession() as s:
                async with s.post(url + "/v1/completions", json={"prompt": "the cat", "max_tokens": 64}) as r:
                    body = await r.json()
                chunks, done = await _stream(url, "/v1/completions", {"prompt": "the cat", "max_tokens": 64})
                assert done
                async with s.post(url + "/v1/chat/completions", json={
                        "messages": [{"role": "user", "content": "hello"}], "max_tokens": 64}) as r:
                    chat = await r.json()
        finally:
            await runner.cleanup()
            eng.stop()
        return body, chunks, chat
    body, chunks, chat = asyncio.run(main())
    assert body["choices"][0]["text"] == want and body["choices"][0]["finish_reason"] == "stop"
    streamed = [c["choices"][0]["text"] for c in chunks if c.get("choices")]
    assert "".join(streamed) == want
    assert all("�" not in t for t in streamed)
    assert chunks[-1]["choices"][0]["finish_reason"] == "stop"
    assert chat["choices"][0]["message"]["content"] == want and "<|eot|>" not in chat["choices"][0]["message"]["content"]


def test_incremental_detokenizer_matches_a_whole_decode(tmp_path):
    from connex_b200.serve.api import HFCodec
    codec = HFCodec(_tiny_bpe_dir(tmp_path))
    text = "a ✓✓ é b — the cat sat 漢字 ok"
    ids = codec.encode(text, add_special=False)
    dt = codec.stream()
    parts = [dt.feed(t) for t in ids] + [dt.flush()]
    assert "".join(parts) == codec.decode(ids) == text
    assert all("�" not in p for p in parts)
