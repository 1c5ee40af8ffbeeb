"""``vllm serve`` (vLLM's OpenAI-compatible server) on the B200 platform, on the CPU.

Starts the server through the plugin's launcher on a tiny random-init Llama with a local
word-level tokenizer, sends token-id and text completion requests over HTTP and checks: the greedy completion equals the framework's own
``LLM.generate``; ``logprobs=0`` returns the sampled token's logprob; requests the platform
cannot serve (``logprobs=2``) are refused with a client error instead of failing the engine.
"""
import json
import os
import signal
import socket
import subprocess
import sys
import time
import urllib.error
import urllib.request

import pytest

pytest.importorskip("vllm")

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CFG = {"architectures": ["LlamaForCausalLM"], "model_type": "llama", "hidden_size": 256,
       "num_hidden_layers": 2, "num_attention_heads": 4, "num_key_value_heads": 2, "head_dim": 64,
       "intermediate_size": 512, "vocab_size": 32000, "rms_norm_eps": 1e-5, "rope_theta": 500000.0,
       "max_position_embeddings": 1024, "torch_dtype": "float32", "tie_word_embeddings": False}


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _post(url, body):
    req = urllib.request.Request(url, data=json.dumps(body).encode(), headers={"Content-Type": "application/json"})
    try:
        with urllib.request.urlopen(req, timeout=120) as r:
            return r.status, json.loads(r.read())
    except urllib.error.HTTPError as e:
        return e.code, json.loads(e.read() or b"{}")


def _tokenizer(d):
    """A word-level tokenizer over the tiny model's vocabulary ("w<id>" words), saved locally."""
    from tokenizers import Tokenizer, decoders, models, pre_tokenizers
    from transformers import PreTrainedTokenizerFast

    vocab = {f"w{i}": i for i in range(31990)}
    vocab.update({"<unk>": 31990, "<s>": 31991, "</s>": 31992})
    tok = Tokenizer(models.WordLevel(vocab=vocab, unk_token="<unk>"))
    tok.pre_tokenizer = pre_tokenizers.WhitespaceSplit()
    tok.decoder = decoders.WordPiece(prefix="##")
    PreTrainedTokenizerFast(tokenizer_object=tok, unk_token="<unk>", bos_token="<s>",
                            eos_token="</s>").save_pretrained(str(d))


def test_vllm_serve_completions(tmp_path):
    (tmp_path / "config.json").write_text(json.dumps(CFG))
    _tokenizer(tmp_path)
    port = _port()
    env = dict(os.environ, PYTHONPATH=ROOT + os.pathsep + os.environ.get("PYTHONPATH", ""))
    cmd = [sys.executable, "-m", "vllm_neuron_b200.vllm_plugin.serve", "--model", str(tmp_path),
           "--dtype", "float32", "--max-model-len", "256", "--max-num-seqs", "4",
           "--max-num-batched-tokens", "64", "--load-format", "dummy", "--enforce-eager", "--seed", "0",
           "--host", "127.0.0.1", "--port", str(port)]
    log = open(tmp_path / "server.log", "w")
    proc = subprocess.Popen(cmd, cwd=str(tmp_path), env=env, stdout=log, stderr=subprocess.STDOUT,
                            start_new_session=True)
    try:
        url = f"http://127.0.0.1:{port}"
        for _ in range(200):
            if proc.poll() is not None:
                break
            try:
                with urllib.request.urlopen(url + "/health", timeout=2) as r:
                    if r.status == 200:
                        break
            except Exception:
                time.sleep(1)
        assert proc.poll() is None, (tmp_path / "server.log").read_text()[-3000:]
        prompt = list(range(1, 21))
        code, res = _post(url + "/v1/completions", {"model": str(tmp_path), "prompt": prompt, "max_tokens": 6,
                                                    "temperature": 0, "ignore_eos": True,
                                                    "return_token_ids": True})
        assert code == 200, res
        got = res["choices"][0].get("token_ids")
        assert res["usage"]["completion_tokens"] == 6 and res["choices"][0]["finish_reason"] == "length"
        # a text prompt, detokenized output and the sampled tokens' logprobs (raw distribution)
        code, res = _post(url + "/v1/completions", {"model": str(tmp_path), "prompt": "w1 w2 w3 w4 w5 w6",
                                                    "max_tokens": 3, "temperature": 0, "ignore_eos": True,
                                                    "logprobs": 0})
        assert code == 200, res
        ch = res["choices"][0]
        lp = ch["logprobs"]["token_logprobs"]
        assert len(lp) == 3 and all(-20.0 < v < 0.0 for v in lp), lp
        assert ch["text"].split() == ch["logprobs"]["tokens"]
        code, res = _post(url + "/v1/completions", {"model": str(tmp_path), "prompt": prompt, "max_tokens": 3,
                                                    "logprobs": 2})
        assert 400 <= code < 500, res
        # the engine is still serving after the refusal
        code, res = _post(url + "/v1/completions", {"model": str(tmp_path), "prompt": prompt[:5], "max_tokens": 2,
                                                    "temperature": 0, "ignore_eos": True})
        assert code == 200, res
    finally:
        try:
            os.killpg(proc.pid, signal.SIGTERM)
            proc.wait(timeout=30)
        except Exception:
            os.killpg(proc.pid, signal.SIGKILL)
        log.close()
    if got is not None:
        from vllm_neuron_b200.engine.sampling_params import SamplingParams
        from vllm_neuron_b200.entrypoints import LLM

        ours = LLM(dict(CFG), max_num_seqs=4, max_model_len=256, max_num_batched_tokens=64, num_gpu_blocks=64,
                   load_format="dummy", device="cpu", dtype="float32", skip_tokenizer_init=True, seed=0)
        ref = ours.generate([prompt], SamplingParams(temperature=0.0, max_tokens=6, ignore_eos=True))
        assert list(got) == list(ref[0].outputs[0].token_ids)
