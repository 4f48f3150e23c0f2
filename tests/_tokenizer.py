"""A small word-level tokenizer with a Qwen-style chat template, saved the way
transformers saves one (tokenizer.json + tokenizer_config.json), so the chat
frontend can be tested without the real Qwen3 tokenizer: word `w<i>` is token
i, the role names and the chat markers follow."""

from __future__ import annotations

from pathlib import Path

TEMPLATE = ("{% for m in messages %}<|im_start|> {{ m['role'] }} {{ m['content'] }} <|im_end|> "
            "{% endfor %}{% if add_generation_prompt %}<|im_start|> assistant "
            "{% if not enable_thinking %}<think> </think> {% endif %}{% endif %}")


def write_tokenizer(model_dir: Path, words: int) -> dict[str, int]:
    """Saves the tokenizer into model_dir; returns the ids of the non-word tokens."""
    from tokenizers import Tokenizer, decoders, models, pre_tokenizers
    from transformers import PreTrainedTokenizerFast

    vocab = {f"w{i}": i for i in range(words)}
    extra = ["<|endoftext|>", "<|im_start|>", "<|im_end|>", "<think>", "</think>",
             "system", "user", "assistant"]
    for j, s in enumerate(extra):
        vocab[s] = words + j
    tok = Tokenizer(models.WordLevel(vocab=vocab, unk_token="<|endoftext|>"))
    tok.pre_tokenizer = pre_tokenizers.WhitespaceSplit()
    tok.decoder = decoders.WordPiece(prefix="##")
    fast = PreTrainedTokenizerFast(tokenizer_object=tok, eos_token="<|im_end|>",
                                   pad_token="<|endoftext|>",
                                   additional_special_tokens=["<|im_start|>", "<|im_end|>"])
    fast.chat_template = TEMPLATE
    fast.save_pretrained(str(model_dir))
    return {s: words + j for j, s in enumerate(extra)}
