// Prompt-lookup speculative decoding (the reference's QWEN3_SPECULATIVE chat
// loop, main_baremetal.c:552-593 and 636-690) over the all-rows forward
// n550_qwen3_forward_rows (qwen3.c:556-566).
//
// Why it pays on the GPU as it does on the AME: a decode step of one token is
// a 1.19 GB weight stream, and verifying k + 1 tokens in one call streams the
// same weights once, so every accepted draft token is a step saved. Drafts come
// from the history itself: the last `ngram` tokens are looked up in the prompt
// and the generated text, newest match first, and the tokens that followed
// that match are proposed. The output is the greedy sequence: a draft token is
// kept only where the model's own argmax at that row equals it.
#include <vector>

#include "common.cuh"

extern "C" {

int n550_lookup_draft(const int32_t *hist, int n_hist, int ngram, int32_t *draft, int max_k) {
    if (n_hist < 0 || ngram < 1 || (n_hist > 0 && !hist) || (max_k > 0 && !draft))
        return N550_ERR_ARG;
    if (max_k <= 0 || n_hist < ngram + 1) return 0;
    const int32_t *tail = hist + n_hist - ngram;
    // newest earlier occurrence of the tail first; it always has a successor
    for (int start = n_hist - ngram - 1; start >= 0; --start) {
        int j = 0;
        while (j < ngram && hist[start + j] == tail[j]) ++j;
        if (j < ngram) continue;
        int k = 0;
        for (int src = start + ngram; k < max_k && src < n_hist; ++src) draft[k++] = hist[src];
        return k;
    }
    return 0;
}

int n550_qwen3_generate_lookup(n550_model_t *m, const int32_t *prompt, int n_prompt, int max_new,
                               int max_draft, int ngram, const int32_t *eos, int n_eos,
                               int32_t *out, int *n_out, n550_spec_stats *stats) {
    if (!m || !prompt || n_prompt < 1 || max_new < 0 || max_draft < 0 || ngram < 1 || n_eos < 0 ||
        (n_eos && !eos) || (max_new && !out) || !n_out)
        return N550_ERR_ARG;
    if (max_draft > N550_ROWS_MAX - 1) max_draft = N550_ROWS_MAX - 1;
    *n_out = 0;
    n550_spec_stats st{};
    auto is_eos = [&](int32_t t) {
        for (int i = 0; i < n_eos; i++)
            if (eos[i] == t) return true;
        return false;
    };
    std::vector<int32_t> hist(prompt, prompt + n_prompt);
    hist.reserve((size_t)n_prompt + max_new);
    // prefill: the prompt's last-token argmax is the first token to emit
    int next = n550_qwen3_forward_batch_host(m, prompt, n_prompt, 0, nullptr);
    if (next < 0) return next;
    n550_model_config cfg{};
    int rc = n550_qwen3_get_config(m, &cfg);
    if (rc) return rc;
    const int budget = cfg.max_len - n_prompt;          // positions left in the KV cache
    const int limit = max_new < budget ? max_new : (budget > 0 ? budget : 0);
    std::vector<int32_t> batch(N550_ROWS_MAX), ids(N550_ROWS_MAX);
    int pos = n_prompt, got = 0;
    while (got < limit) {
        if (is_eos(next)) break;
        int k = n550_lookup_draft(hist.data(), (int)hist.size(), ngram, batch.data() + 1, max_draft);
        if (k < 0) return k;
        if (k > limit - got - 1) k = limit - got - 1;      // no drafts past the budget
        if (k < 0) k = 0;
        batch[0] = next;
        // row j's argmax is the token that follows batch[0..j]: it verifies batch[j + 1]
        rc = n550_qwen3_forward_rows_host(m, batch.data(), k + 1, pos, ids.data(), nullptr);
        if (rc) return rc;
        st.rounds++;
        st.drafted += k;
        out[got++] = next;
        hist.push_back(next);
        int kept = 1;                      // positions of this call that stay in the cache
        bool stop = false;
        for (int j = 0; j < k && got < limit; j++) {
            const int32_t pred = ids[j];
            if (pred != batch[j + 1] || is_eos(pred)) {
                if (pred == batch[j + 1]) st.accepted++;
                next = pred;
                stop = true;
                break;
            }
            st.accepted++;
            out[got++] = pred;
            hist.push_back(pred);
            kept++;
        }
        if (!stop) next = ids[k];          // every draft kept (or none made): the last row's choice
        pos += kept;                       // cache rows past `pos` are rewritten by the next call
    }
    *n_out = got;
    if (stats) *stats = st;
    return N550_OK;
}

int n550_qwen3_chat(n550_model_t *m, const n550_tok_t *tok, const char *prompt, size_t len,
                    int max_new, int max_draft, char *text, size_t max_text, int32_t *ids,
                    int *n_ids) {
    if (!m || !tok || (len && !prompt) || max_new < 0 || !text || !max_text || (max_new && !ids) ||
        !n_ids)
        return N550_ERR_ARG;
    n550_model_config cfg{};
    int rc = n550_qwen3_get_config(m, &cfg);
    if (rc) return rc;
    std::vector<int32_t> in(cfg.max_tokens);
    const int n_in = n550_chat_encode(tok, prompt, len, in.data(), cfg.max_tokens);
    if (n_in < 0) return n_in;
    if (n_in == 0) return N550_ERR_ARG;
    const int32_t eos[2] = {151645, 151643};          // QWEN3_EOS_TOKEN_ID_0 / _1
    rc = n550_qwen3_generate_lookup(m, in.data(), n_in, max_new, max_draft, 3, eos, 2, ids, n_ids,
                                    nullptr);
    if (rc) return rc;
    return n550_tok_decode(tok, ids, *n_ids, text, max_text);
}

}  // extern "C"
