"""Compose reports: ``compose_report.json``, ``BUILD.md`` (with the population table) and a ``README.md`` model card.

(reference: src/granite_switch/composer/reporting/compose_report.py:88,
model_card.py:331.) The report records, per adapter slot: name, technology,
kind, rank, control token, substitute, target module groups and source.
"""
from __future__ import annotations

import json
import os
import time


def adapter_rows(config, adapters):
    off = len(config.adapter_token_ids or []) - config.num_adapters
    rows = []
    for i, a in enumerate(adapters):
        rows.append({
            "adapter_index": i + 1, "name": a.name, "technology": a.technology, "kind": a.kind,
            "rank": (config.adapter_ranks or [None] * config.num_adapters)[i],
            "control_token": f"<|{a.name}|>", "control_token_id": config.adapter_token_ids[i + off],
            "substitute_token_id": config.adapter_substitute_token_ids[i + off],
            "target_groups": sorted(a.target_groups()), "source": a.source,
        })
    return rows


def write_reports(out_dir, config, adapters, base_model: str, seconds: float) -> None:
    rows = adapter_rows(config, adapters)
    report = {"base_model": base_model, "num_adapters": config.num_adapters,
              "num_decoder_layers": config.num_decoder_layers, "vocab_size": config.vocab_size,
              "lora_target_modules": config.lora_target_modules, "max_lora_rank": config.max_lora_rank,
              "base_reset": config.has_base_reset, "dual_stream": config.dual_stream,
              "asr_enabled": config.asr_enabled, "compose_seconds": round(seconds, 2),
              "validation": getattr(config, "compose_validation", None),
              "created": time.strftime("%Y-%m-%dT%H:%M:%SZ", time.gmtime()), "adapters": rows}
    with open(os.path.join(out_dir, "compose_report.json"), "w") as f:
        json.dump(report, f, indent=2)
    lines = [f"# Granite Switch checkpoint", "", f"Base model: `{base_model}`", "",
             f"{config.num_adapters} adapter slots over {config.num_decoder_layers} decoder layers; "
             f"LoRA targets: {', '.join(config.lora_target_modules) or 'none'}.", "",
             "| # | adapter | technology | kind | rank | control token (id) |", "|---|---|---|---|---|---|"]
    for r in rows:
        lines.append(f"| {r['adapter_index']} | {r['name']} | {r['technology']} | {r['kind']} | {r['rank']} | "
                     f"`{r['control_token']}` ({r['control_token_id']}) |")
    lines += ["", "Select an adapter by rendering the chat template with `adapter_name=<name>`, "
                  "and send prompts as token ids so the prefix cache can be shared across adapters.", ""]
    pop = population_table(config)
    if pop:
        lines += ["## Population (decoder layers holding each adapter's weights)", "", *pop, ""]
    with open(os.path.join(out_dir, "BUILD.md"), "w") as f:
        f.write("\n".join(lines))
    write_model_card(out_dir, config, rows, base_model)


def population_table(config) -> list[str]:
    """Markdown table: for each adapter, in how many decoder layers each module group is populated
    (reference: src/granite_switch/composer/reporting/population_table.py:10)."""
    v = getattr(config, "compose_validation", None) or {}
    pop = v.get("layers_populated") or {}
    if not pop:
        return []
    groups = sorted({g for row in pop.values() for g in row})
    n = config.num_decoder_layers
    out = ["| adapter | " + " | ".join(groups) + " |", "|---|" + "---|" * len(groups)]
    for name, row in pop.items():
        out.append(f"| {name} | " + " | ".join(f"{row.get(g, 0)}/{n}" for g in groups) + " |")
    return out


def write_model_card(out_dir, config, rows, base_model: str) -> None:
    """``README.md``: what the checkpoint holds and how to select an adapter
    (reference: src/granite_switch/composer/reporting/model_card.py:233-331)."""
    kinds = {r["name"]: ("probe" if r["kind"] == "probe" else r["technology"]) for r in rows}
    lines = ["---", "library_name: granite_switch_b200", f"base_model: {base_model}", "tags:", "- granite-switch",
             "- lora", "---", "", "# Granite Switch checkpoint", "",
             f"One set of base weights (`{base_model}`) serving {config.num_adapters} adapters, selected per "
             f"token by control tokens in the prompt. Shadow Residual: {bool(config.dual_stream)}. "
             f"Base-reset token: {bool(config.has_base_reset)}. Audio cascade: {bool(config.asr_enabled)}.", "",
             "## Adapters", "", "| adapter | kind | rank | control token |", "|---|---|---|---|"]
    for r in rows:
        lines.append(f"| {r['name']} | {kinds[r['name']]} | {r['rank']} | `{r['control_token']}` |")
    example = rows[0]["name"] if rows else "ADAPTER"
    lines += ["", "## Usage", "", "```python",
              "from transformers import AutoTokenizer",
              "from granite_switch_b200.engine import LLM, SamplingParams", "",
              "tok = AutoTokenizer.from_pretrained(PATH)",
              f"ids = tok.apply_chat_template(messages, add_generation_prompt=True, adapter_name={example!r})",
              "out = LLM(PATH).generate([ids], SamplingParams(max_tokens=256))", "```", "",
              "LoRA adapters apply to the whole prompt; aLoRA adapters activate at their invocation text, so "
              "the prompt before it shares the prefix cache with every other adapter; Shadow Residual "
              "adapters take over at the generation prompt; probes return a verdict at the last token.", ""]
    with open(os.path.join(out_dir, "README.md"), "w") as f:
        f.write("\n".join(lines))
