"""Known-answer tests derived by hand from src/nimllm/sampler.nim (reference
repository). Each case cites the lines that determine its answer; the
expected id was worked out on paper from those lines, not computed by any of
the restatements. Shared by the CPU oracle tests and the GPU parity tests.

A case: (name, logits, params tuple, history, bias dict, uniform, expected id)
params tuple = (temperature, top_p, min_p, repeat_penalty, presence_penalty,
                frequency_penalty, top_k, repeat_last_n)
"""
import math

INF = math.inf
G = (0.0, 1.0, 0.0, 1.0, 0.0, 0.0, 0, 64)       # greedy, nothing else
S = (1.0, 1.0, 0.0, 1.0, 0.0, 0.0, 0, 64)       # T=1, full sort, no cut-offs


def P(**kw):
    names = ["temperature", "top_p", "min_p", "repeat_penalty", "presence_penalty",
             "frequency_penalty", "top_k", "repeat_last_n"]
    base = dict(zip(names, S))
    base.update(kw)
    return tuple(base[n] for n in names)


KATS = [
    # argmax keeps the first index of the maximum (:47-48, strict `>`)
    ("argmax_tie_lowest_index", [1.0, 3.0, 3.0, 2.0], G, [], {}, 0.5, 1),
    # a NaN never wins unless it is at index 0 (:48 compares with `>`)
    ("argmax_nan_ignored", [1.0, math.nan, 2.0], G, [], {}, 0.5, 2),
    ("argmax_nan_at_zero", [math.nan, 5.0, 6.0], G, [], {}, 0.5, 0),
    # heap (k=2) on [1,1,2]: (1,0) is evicted by (2,2), (1,1) survives; order
    # after reverse is [2, 1]; probs [0.731, 0.269]; u=0.9 -> second (:88-95)
    ("heap_tie_keeps_higher_index", [1.0, 1.0, 2.0], P(top_k=2), [], {}, 0.9, 1),
    # full stable sort (k=0) on the same logits: [2, 0, 1]; probs
    # [0.576, 0.212, 0.212]; u=0.7 -> r=0.124 after the first -> index 0 (:97)
    ("full_sort_tie_ascending_index", [1.0, 1.0, 2.0], S, [], {}, 0.7, 0),
    # top_k >= V takes the full-sort path (:85-86)
    ("topk_ge_vocab_is_full_sort", [1.0, 1.0, 2.0], P(top_k=3), [], {}, 0.7, 0),
    ("topk_gt_vocab_is_full_sort", [1.0, 1.0, 2.0], P(top_k=9), [], {}, 0.7, 0),
    # uniform 0: r = 0, the first subtraction makes it negative -> idx[0] (:117-120)
    ("uniform_zero_takes_first", [0.0, 1.0, 0.5], S, [], {}, 0.0, 1),
    # top-p=0.5 over probs [0.576,0.212,0.212] keeps one candidate (:103-108)
    ("top_p_cuts_to_one", [1.0, 1.0, 2.0], P(top_p=0.5), [], {}, 0.99, 2),
    # top_p = 0 disables the cut (:103), so u=0.99 reaches the last candidate
    ("top_p_zero_disables", [1.0, 1.0, 2.0], P(top_p=0.0), [], {}, 0.99, 1),
    ("top_p_one_disables", [1.0, 1.0, 2.0], P(top_p=1.0), [], {}, 0.99, 1),
    # min-p 0.5: thr = 0.576*0.5 = 0.288 > 0.212 -> only the first survives (:110-114)
    ("min_p_cuts", [1.0, 1.0, 2.0], P(min_p=0.5), [], {}, 0.99, 2),
    # repeat penalty divides a positive logit: 2/2 = 1 < 1.5 -> token 1 wins greedy (:72)
    ("repeat_penalty_divides_positive", [2.0, 1.5], (0.0, 1.0, 0.0, 2.0, 0.0, 0.0, 0, 64), [0], {}, 0.5, 1),
    # ... and multiplies a negative one: -1*2 = -2 < -1.5 -> token 1 (:73)
    ("repeat_penalty_multiplies_negative", [-1.0, -1.5], (0.0, 1.0, 0.0, 2.0, 0.0, 0.0, 0, 64), [0], {}, 0.5, 1),
    # zero takes the multiply branch and stays 0; presence 0.5 makes it -0.5 (:73-74)
    ("penalty_zero_logit_and_presence", [0.0, -0.25], (0.0, 1.0, 0.0, 2.0, 0.5, 0.0, 0, 64), [0], {}, 0.5, 1),
    # frequency: count 3 * 0.5 = 1.5 subtracted from 2 -> 0.5 < 1 (:74)
    ("frequency_penalty_counts", [2.0, 1.0], (0.0, 1.0, 0.0, 1.0, 0.0, 0.5, 0, 64), [0, 0, 0], {}, 0.5, 1),
    # window of the last 1 id: only id 1 is penalised, id 0 keeps 2.0 (:67)
    ("repeat_last_n_window", [2.0, 1.9], (0.0, 1.0, 0.0, 1.0, 1.0, 0.0, 0, 1), [0, 1], {}, 0.5, 0),
    # repeat_last_n <= 0: the whole history counts, so id 0 (first in the
    # history) drops to 1.0 < 1.9; a window of the last id would leave it (:67)
    ("repeat_last_n_zero_whole_history", [2.0, 1.9], (0.0, 1.0, 0.0, 1.0, 1.0, 0.0, 0, 0), [0, 2, 2], {}, 0.5, 1),
    ("repeat_last_n_negative_whole_history", [2.0, 1.5], (0.0, 1.0, 0.0, 1.0, 1.0, 0.0, 0, -3), [0, 5], {}, 0.5, 1),
    # ids outside [0, V) in history and bias are ignored (:70, :76)
    ("out_of_range_ids_ignored", [1.0, 2.0], (0.0, 1.0, 0.0, 1.0, 5.0, 0.0, 0, 64), [-1, 2, 7], {-4: 9.0, 2: 9.0}, 0.5, 1),
    # rep=1, pres=0, freq=0: the penalty block is skipped entirely (:64-65)
    ("penalties_off_with_history", [1.0, 2.0], (0.0, 1.0, 0.0, 1.0, 0.0, 0.0, 0, 64), [1, 1], {}, 0.5, 1),
    # bias is added after the penalty: (2/2) + 0.75 = 1.75 > 1.5 (:72, :76)
    ("bias_after_penalty", [2.0, 1.5], (0.0, 1.0, 0.0, 2.0, 0.0, 0.0, 0, 64), [0], {0: 0.75}, 0.5, 0),
    # -Inf bias forbids a token even when it had the largest logit
    ("neg_inf_bias_forbids", [5.0, 1.0, 0.0], S, [], {0: -INF}, 0.9999, 2),
    # temperature scales before the heap: T=0.5 -> [2,4,6]; k=1 keeps index 2
    ("temperature_then_topk1", [1.0, 2.0, 3.0], P(temperature=0.5, top_k=1), [], {}, 0.99, 2),
]
