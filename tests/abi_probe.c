/* Prints the layout of the EdgeCore ABI structs as JSON.  Compiled by the
 * tests against include/edgecore.h and, when generating the golden layout,
 * against the reference header, to prove the two are layout-identical. */
#include <stddef.h>
#include <stdio.h>
#include "edgecore.h"

#define F(T, f) printf("  \"%s.%s\": [%zu, %zu],\n", #T, #f, offsetof(T, f), sizeof(((T *)0)->f))

int main(void)
{
    printf("{\n");
    printf("  \"sizeof.GPT2\": %zu,\n  \"sizeof.Tokenizer\": %zu,\n  \"sizeof.EcmTensor\": %zu,\n"
           "  \"sizeof.LayerW\": %zu,\n", sizeof(GPT2), sizeof(Tokenizer), sizeof(EcmTensor),
           sizeof(struct LayerW));
    F(GPT2, model_name); F(GPT2, n_layer); F(GPT2, n_head); F(GPT2, n_embd); F(GPT2, n_ctx);
    F(GPT2, vocab); F(GPT2, n_kv_head); F(GPT2, n_kv_embd); F(GPT2, intermediate); F(GPT2, head_dim);
    F(GPT2, arch); F(GPT2, n_params); F(GPT2, eps); F(GPT2, rope_theta); F(GPT2, rope_type);
    F(GPT2, yarn_factor); F(GPT2, yarn_orig_max); F(GPT2, yarn_attention_factor);
    F(GPT2, sliding_window); F(GPT2, tie_word_embeddings); F(GPT2, eos_token_id); F(GPT2, wte);
    F(GPT2, wpe); F(GPT2, lw); F(GPT2, lnf_g); F(GPT2, lnf_b); F(GPT2, lm_head); F(GPT2, precision);
    F(GPT2, k_cache); F(GPT2, v_cache); F(GPT2, batch_cap); F(GPT2, max_ctx); F(GPT2, ws_x);
    F(GPT2, ws_tmp); F(GPT2, ws_qkv); F(GPT2, ws_attn); F(GPT2, ws_scores); F(GPT2, ws_q);
    F(GPT2, ws_qs); F(GPT2, ws_q_cols); F(GPT2, tok); F(GPT2, file_data); F(GPT2, file_size);
    F(GPT2, file_mapped);
    F(struct LayerW, ln1_g); F(struct LayerW, attn_w); F(struct LayerW, fc2_b); F(struct LayerW, q_w);
    F(struct LayerW, o_s); F(struct LayerW, v_b); F(struct LayerW, gate_w); F(struct LayerW, down_b);
    F(Tokenizer, id_to_token); F(Tokenizer, merge_m); F(Tokenizer, n_merges); F(Tokenizer, eos_id);
    F(Tokenizer, sp_tok); F(Tokenizer, n_sp);
    F(EcmTensor, name); F(EcmTensor, dtype); F(EcmTensor, nelems); F(EcmTensor, bytes);
    F(EcmTensor, offset); F(EcmTensor, dims); F(EcmTensor, ndims);
    printf("  \"end\": 0\n}\n");
    return 0;
}
