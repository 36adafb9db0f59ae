"""DSpark semantics on the CPU oracle (V4.1 tiny config, Engram included):
speculative decoding with honest acceptance emits exactly the greedy stream
(the reference's lossless check, verify_dspark_speculative.py Check 1), and
forced acceptance emits block-size tokens per round."""

import torch

from dsv4_flash_deployment_b200.config import v41_tiny_config
from dsv4_flash_deployment_b200.io.checkpoint_spec import make_random_weights
from dsv4_flash_deployment_b200.ref.model import RefModel


def _spec(ref, cfg, prompt, n_new, force=None):
    st = ref.new_state(1)
    ref.dspark_state_init(st)
    mh, lg = [], None
    for t in prompt:
        lg, h = ref.step(torch.tensor([t]), st)
        mh.append(h)
    out = [int(lg.argmax(-1)[0])]
    start, rows = 0, torch.stack(mh, 1)
    rounds = []
    while len(out) < n_new:
        toks, logits, conf = ref.draft(torch.tensor([out[-1]]), rows, start, st)
        assert toks.shape == (1, cfg.dspark_block_size + 1) and conf.shape == (1, cfg.dspark_block_size)
        res = ref.verify(toks[:, :cfg.dspark_block_size], st, force_accept=force)
        rounds.append(res["num_accepted"])
        start = st.pos - (res["num_accepted"] + 1)
        rows = res["main_hidden"]
        out.extend(res["emitted"])
    return out[:n_new], rounds


def test_spec_is_lossless_and_forced_blocks():
    cfg = v41_tiny_config()
    w = make_random_weights(cfg, seed=2)
    ref = RefModel(cfg, w, max_seq_len=96)
    prompt = torch.randint(0, cfg.vocab_size, (10,), generator=torch.Generator().manual_seed(3)).tolist()
    greedy, _ = ref.generate(torch.tensor([prompt]), 12)
    spec, rounds = _spec(ref, cfg, prompt, 12)
    assert spec == greedy[0].tolist()
    forced, rf = _spec(ref, cfg, prompt, 12, force=cfg.dspark_block_size - 1)
    assert all(r == cfg.dspark_block_size - 1 for r in rf)
    assert forced[0] == greedy[0, 0].item() and len(rf) == 3   # 1 + 5 + 5 + (1) tokens
