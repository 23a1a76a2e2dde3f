"""Compose reports: ``compose_report.json`` and a ``BUILD.md`` model card.

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
    with open(os.path.join(out_dir, "BUILD.md"), "w") as f:
        f.write("\n".join(lines))
