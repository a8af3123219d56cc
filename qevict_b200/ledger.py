"""``get_ledger_data`` of the reference (src/models/kv_cache/ledger.py:16-44):
the active rows of a token ledger split into named columns, on the host."""


def get_ledger_data(global_token_counter, token_ledger, num_heads):
    n = int(global_token_counter)
    active = token_ledger[:n].detach().cpu()
    return {
        "global_id": active[:, 0].long(),
        "layer_id": active[:, 1].long(),
        "physical_id": active[:, 2:2 + num_heads].long(),
        "attention_score": active[:, 2 + num_heads:2 + 2 * num_heads],
    }
