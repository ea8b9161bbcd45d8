"""The LONGER encoder against the reference's own ``LongerSequenceEncoder`` (CPU, fp32):
identical weights and inputs (event tokens, user and candidate global tokens, padded
sequences, token merging with inner blocks) give the same flattened output
(``[user globals; candidate globals; recent]``)."""

import pytest
import torch

from baseline import install

pytestmark = pytest.mark.skipif(not install.installed(), reason="reference not installed under baseline/_ref")


def _ours(merge, inner, self_layers, cand, d=8, heads=2, R=6, L=30):
    from mdl_b200.config.loader import app_config_from_mapping
    from mdl_b200.data.baseline_configs import scaled_config
    from mdl_b200.models.factory import build_model

    m, _ = scaled_config(5, 1e-4, num_fields=12, batch=8, seq_len=L, min_len=2, query_tokens=R,
                         self_layers=self_layers, d=d, heads=heads, sequence_head="none", ns_tokens=4)
    m["sequences"][0].update({"longer_candidate_global_tokens": cand, "longer_token_merge": merge,
                              "longer_inner_layers": inner})
    torch.manual_seed(0)
    return build_model(app_config_from_mapping(m), device="cpu", base_seed=1).longer


@pytest.mark.parametrize("merge,inner,self_layers,cand", [(1, 0, 2, 1), (2, 1, 1, 2), (3, 0, 0, 1)])
def test_longer_encoder_matches_reference(merge, inner, self_layers, cand):
    from baseline import reference_harness as rh

    rh._import_reference()
    from src.model import LongerSequenceEncoder

    enc = _ours(merge, inner, self_layers, cand)
    Gu, Gc, R, L, Din, D = enc.Gu, enc.Gc, enc.R, enc.L, enc.Din, enc.D
    ref = LongerSequenceEncoder(Din, enc.heads, enc.inner[0].hidden_dim if inner else enc.step.hidden, R,
                                self_layers, Gu + Gc, merge, inner, user_global_tokens=Gu,
                                attention_backend="sdpa")
    sd = {}
    sd.update(enc.cross.reference_state_dict("cross_block."))
    for i, blk in enumerate(enc.selfs):
        sd.update(blk.reference_state_dict(f"self_blocks.{i}."))
    for i, blk in enumerate(enc.inner):
        sd.update(blk.reference_state_dict(f"token_merger.inner_blocks.{i}."))
    missing, unexpected = ref.load_state_dict(sd, strict=False)
    assert not unexpected and not [k for k in missing if "ffn" in k or "norm" in k or "projection" in k], missing
    ref.eval()
    torch.manual_seed(3)
    B = 5
    tokens = torch.randn(B, L, Din)
    lengths = torch.tensor([L, 17, 4, 1, 0])
    valid = torch.arange(L).view(1, L) >= (L - lengths).view(B, 1)
    user = torch.randn(B, Gu, D)
    cand = torch.randn(B, Gc, D)
    with torch.no_grad():
        want = ref(tokens, valid, cand, user_global_tokens=user)
        got = enc(None, lengths, None, None, False, tokens=tokens, user_tokens=user, cand_tokens=cand)
        got = type(enc).reference_order(got, enc.G).reshape(B, -1)
    torch.testing.assert_close(got, want, atol=2e-5, rtol=2e-5)
