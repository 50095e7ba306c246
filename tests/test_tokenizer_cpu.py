"""Hugging Face tokenizer from a checkpoint directory: chat prompts carry the
template's BOS exactly once."""
import json


def _make_tokenizer_dir(d):
    from tokenizers import Tokenizer, models, pre_tokenizers, processors
    vocab = {"<bos>": 0, "<eos>": 1, "<unk>": 2, "hello": 3, "world": 4, "user": 5, "assistant": 6, ":": 7}
    tk = Tokenizer(models.WordLevel(vocab, unk_token="<unk>"))
    tk.pre_tokenizer = pre_tokenizers.WhitespaceSplit()
    # plain encodes get a BOS, as DeepSeek's tokenizer does
    tk.post_processor = processors.TemplateProcessing(single="<bos> $A", special_tokens=[("<bos>", 0)])
    tk.save(str(d / "tokenizer.json"))
    tmpl = ("{{ bos_token }}{% for m in messages %}{{ m['role'] }} : {{ m['content'] }} {% endfor %}"
            "{% if add_generation_prompt %}assistant : {% endif %}")
    (d / "tokenizer_config.json").write_text(json.dumps({
        "tokenizer_class": "PreTrainedTokenizerFast", "bos_token": "<bos>", "eos_token": "<eos>",
        "unk_token": "<unk>", "add_bos_token": True, "chat_template": tmpl}))


def test_hf_chat_prompt_has_one_bos(tmp_path):
    from b200ds.engine.tokenizer import HFTokenizer, load_tokenizer
    _make_tokenizer_dir(tmp_path)
    tok = load_tokenizer(str(tmp_path))
    assert isinstance(tok, HFTokenizer) and tok.eos_token_id == 1
    ids = tok.encode_chat([{"role": "user", "content": "hello world"}])
    assert ids.count(0) == 1 and ids[0] == 0
    assert ids[1:] == [5, 7, 3, 4, 6, 7]
    assert tok.encode("hello")[0] == 0                            # plain text: BOS added
    assert tok.encode(tok.apply_chat_template([{"role": "user", "content": "hello"}]))[:2] == [0, 0]
    assert tok.decode([3, 4, 1]) == "hello world"
