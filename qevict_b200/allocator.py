"""Token-budget allocation of the Sticky-KV cache (host arithmetic).

``compute_budget`` keeps the reference's signature and result type
(``compute_budget`` / ``BudgetResult``, src/models/kv_cache/allocator.py:17-107):
sinks first, then the local zone, then the rest split between full-precision
sticky windows and the quantised Q-cache, with the Q share scaled by the
compression ratio of the code width and both window counts rounded up.
"""

from collections import namedtuple

BudgetResult = namedtuple("BudgetResult", ["local_num", "k_windows", "q_windows_count", "q_num", "quant_bytes_len"])


def compute_budget(total_cache_ratio, sink_tokens, use_fixed_local_tokens, local_num_tokens, local_cache_ratio,
                   q_ratio, quant_bit_width, head_dim, omega, new_tokens, max_tokens, layer_idx):
    """Window budget for a prompt of ``new_tokens`` followed by up to ``max_tokens`` generated ones.

    Returns BudgetResult(local_num, k_windows, q_windows_count, q_num, quant_bytes_len):
    local-zone tokens, sticky windows, Q-cache windows, the full-precision-equivalent
    tokens the Q-cache occupies, and bytes per quantised token row.
    """
    budget = (new_tokens + max_tokens) * total_cache_ratio // 100
    left = max(0, budget - sink_tokens)
    want_local = local_num_tokens if use_fixed_local_tokens else budget * local_cache_ratio // 100
    local_num = min(want_local, left)
    left = max(0, left - local_num)
    # bytes per token row: 2*D at full precision, D (INT8) or D/2 (INT4) quantised
    ratio = (2 * head_dim) / (head_dim if quant_bit_width == 8 else head_dim / 2.0)
    sticky_tokens = left * (100 - q_ratio) // 100
    q_tokens = int((left - sticky_tokens) * ratio)
    k_windows = -(-sticky_tokens // omega)
    q_windows = -(-q_tokens // omega)
    q_num = int((q_windows * omega) / ratio)
    if k_windows == 0:
        print(f"WARNING [Layer {layer_idx}]: k_windows=0 -- insufficient budget for sticky windows "
              f"(budget={budget}, local={local_num}, sink={sink_tokens}, q_windows={q_windows}). "
              f"Eviction is effectively disabled.")
    qbytes = head_dim if quant_bit_width == 8 else head_dim // 2
    return BudgetResult(local_num, k_windows, q_windows, q_num, qbytes)
