"""vLLM platform plugin (CPU): registration, and vLLM's own engine (``vllm.LLM``: scheduler,
KV-block manager, prefix caching, chunked prefill) driving this framework's worker, which must
produce the same greedy tokens as the framework's own ``LLM.generate``."""
import json
import os
import subprocess
import sys
import textwrap

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CFG = {"architectures": ["LlamaForCausalLM"], "model_type": "llama", "hidden_size": 256,
       "num_hidden_layers": 2, "num_attention_heads": 4, "num_key_value_heads": 2, "head_dim": 64,
       "intermediate_size": 512, "vocab_size": 32000, "rms_norm_eps": 1e-5, "rope_theta": 500000.0,
       "max_position_embeddings": 1024, "torch_dtype": "float32", "tie_word_embeddings": False}

vllm = pytest.importorskip("vllm")


def test_register(monkeypatch):
    from vllm_neuron_b200.vllm_plugin import PLATFORM_CLS, register

    monkeypatch.setenv("VLLM_B200_PLUGIN", "1")
    assert register() == PLATFORM_CLS
    monkeypatch.setenv("VLLM_B200_PLUGIN", "0")
    assert register() is None
    with open(os.path.join(ROOT, "setup.py")) as f:
        assert "vllm.platform_plugins" in f.read()


@pytest.mark.parametrize("async_sched", [False, True])
def test_vllm_engine_through_b200_worker(tmp_path, async_sched):
    """vLLM's LLM on the B200 worker equals the framework's own engine (greedy), with vLLM's
    synchronous and asynchronous scheduling (the worker then launches each step before the
    previous one's tokens are back, reading them on the device)."""
    (tmp_path / "config.json").write_text(json.dumps(CFG))
    script = textwrap.dedent(f"""
        import json, os, sys
        sys.path.insert(0, {ROOT!r})
        os.environ["VLLM_ENABLE_V1_MULTIPROCESSING"] = "0"
        import torch
        import vllm.platforms as vp
        from vllm_neuron_b200.vllm_plugin.platform import B200Platform
        vp._current_platform = B200Platform()
        from vllm import LLM, SamplingParams
        g = torch.Generator().manual_seed(0)
        prompts = [torch.randint(0, 32000, (n,), generator=g).tolist() for n in (32, 40, 7, 100)]
        prompts.append(prompts[0][:20] + [5, 6, 7])  # shares a cached prefix block with prompt 0
        llm = LLM(model={str(tmp_path)!r}, skip_tokenizer_init=True, dtype="float32", max_model_len=256,
                  max_num_seqs=4, max_num_batched_tokens=64, load_format="dummy", seed=0, block_size=16,
                  enforce_eager=True, async_scheduling={async_sched!r})
        assert llm.llm_engine.vllm_config.scheduler_config.async_scheduling == {async_sched!r}
        outs = llm.generate([{{"prompt_token_ids": p}} for p in prompts],
                            SamplingParams(max_tokens=12, temperature=0.0, ignore_eos=True))
        got = [list(o.outputs[0].token_ids) for o in outs]
        from vllm_neuron_b200.engine.sampling_params import SamplingParams as SP
        from vllm_neuron_b200.entrypoints import LLM as B200LLM
        ours = B200LLM({CFG!r}, max_num_seqs=4, max_model_len=256, max_num_batched_tokens=64,
                       num_gpu_blocks=128, load_format="dummy", device="cpu", dtype="float32",
                       skip_tokenizer_init=True, seed=0)
        ref = [list(o.outputs[0].token_ids) for o in
               ours.generate(prompts, SP(temperature=0.0, max_tokens=12, ignore_eos=True))]
        print("RESULT" + json.dumps({{"got": got, "ref": ref}}))
    """)
    env = dict(os.environ, VLLM_B200_PLUGIN="1")
    p = subprocess.run([sys.executable, "-c", script], capture_output=True, text=True, timeout=600,
                       cwd=str(tmp_path), env=env)
    lines = [l for l in p.stdout.splitlines() if l.startswith("RESULT")]
    assert p.returncode == 0 and lines, p.stderr[-4000:]
    res = json.loads(lines[-1][len("RESULT"):])
    assert all(len(t) == 12 for t in res["got"])
    assert res["got"] == res["ref"]


def test_vllm_tp2_mp_executor_gloo(tmp_path):
    """vLLM's multiprocess executor with two B200 workers (TP = 2 over gloo on the CPU, each
    loading its shard of one saved checkpoint) equals the framework's own single-rank engine
    (greedy)."""
    from tests._tiny import tiny_llama_checkpoint

    ckpt, _ = tiny_llama_checkpoint()
    script = textwrap.dedent(f"""
        import json, os, sys
        sys.path.insert(0, {ROOT!r})
        import torch
        import vllm.platforms as vp
        from vllm_neuron_b200.vllm_plugin.platform import B200Platform
        vp._current_platform = B200Platform()
        from vllm import LLM, SamplingParams
        if __name__ == "__main__":
            g = torch.Generator().manual_seed(0)
            prompts = [torch.randint(0, 32000, (n,), generator=g).tolist() for n in (32, 40, 7)]
            llm = LLM(model={ckpt!r}, skip_tokenizer_init=True, dtype="float32", max_model_len=256,
                      max_num_seqs=4, max_num_batched_tokens=64, seed=0, block_size=16,
                      enforce_eager=True, tensor_parallel_size=2, distributed_executor_backend="mp")
            outs = llm.generate([{{"prompt_token_ids": p}} for p in prompts],
                                SamplingParams(max_tokens=8, temperature=0.0, ignore_eos=True))
            got = [list(o.outputs[0].token_ids) for o in outs]
            from vllm_neuron_b200.engine.sampling_params import SamplingParams as SP
            from vllm_neuron_b200.entrypoints import LLM as B200LLM
            ours = B200LLM({ckpt!r}, max_num_seqs=4, max_model_len=256, max_num_batched_tokens=64,
                           num_gpu_blocks=128, device="cpu", dtype="float32", skip_tokenizer_init=True, seed=0)
            ref = [list(o.outputs[0].token_ids) for o in
                   ours.generate(prompts, SP(temperature=0.0, max_tokens=8, ignore_eos=True))]
            print("RESULT" + json.dumps({{"got": got, "ref": ref}}), flush=True)
    """)
    (tmp_path / "run_tp2.py").write_text(script)
    env = dict(os.environ, VLLM_B200_PLUGIN="1", MASTER_ADDR="127.0.0.1", VLLM_HOST_IP="127.0.0.1",
               VLLM_WORKER_MULTIPROC_METHOD="spawn")
    p = subprocess.run([sys.executable, str(tmp_path / "run_tp2.py")], capture_output=True, text=True,
                       timeout=600, cwd=str(tmp_path), env=env)
    lines = [l for l in p.stdout.splitlines() if l.startswith("RESULT")]
    assert lines, (p.stdout[-2000:], p.stderr[-4000:])
    res = json.loads(lines[-1][len("RESULT"):])
    assert all(len(t) == 8 for t in res["got"])
    assert res["got"] == res["ref"]
