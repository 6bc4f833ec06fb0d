"""Token loops around the megakernel (`megakernels/generators.py` of
epic-kernel, :11-166).

`MK_Generator.run` does per token what the reference does: embed the input
token into `hidden_states`, reset the barrier counters, zero the logits, launch
the megakernel, and take the argmax of the logits, all on the current stream
with no host synchronisation. With an interpreter that supports the fused
step (the Llama engine), the gather and the argmax run inside the megakernel
and a step is one barrier reset plus one launch.
"""

import torch
from torch import Tensor

from megakernels.mk import MK_Interpreter
from megakernels.model_types import BatchState
from megakernels.scheduler import Schedule


class Generator:
    def generate(self, output_tokens: Tensor, prompt_len: int, ntok: int,
                 ntok_already_generated: int = 1):
        raise NotImplementedError

    def generate_with_eos(self, output_tokens: Tensor, prompt_len: int, ntok: int,
                          eos_token_check_interval: int, eos_token_ids: list[int]):
        """Generate in chunks, checking for EOS between chunks. Returns (pos of
        the first eos token, tokens generated)."""
        assert output_tokens.shape[0] == 1, "batch size must be 1"
        for done in range(1, ntok, eos_token_check_interval):
            chunk = min(eos_token_check_interval, ntok - done)
            self.generate(output_tokens, prompt_len=prompt_len, ntok=chunk,
                          ntok_already_generated=done)
            for j, token in enumerate(output_tokens[0, done : done + chunk].cpu()):
                if token in eos_token_ids:
                    return done + j, done + chunk - 1
        return ntok, ntok - 1


class MK_Generator(Generator):
    def __init__(self, model, interpreter: MK_Interpreter, schedule: Schedule,
                 barrier_fill_val: int = 0, skip_mk: bool = False, skip_rest: bool = False):
        self.model = model
        self.interpreter = interpreter
        self.schedule = schedule
        self.barrier_fill_val = barrier_fill_val
        self.skip_mk = skip_mk
        self.skip_rest = skip_rest
        self.fill()

    def _fused_step(self) -> bool:
        if self.skip_mk or self.skip_rest or not getattr(self.interpreter, "supports_fused_step", False):
            return False
        if getattr(self.schedule.globs, "lm_head_instructions", 0) < 1:
            return False
        if not hasattr(self, "_tokens"):
            self._tokens = torch.zeros(2, 1, dtype=torch.int64, device=self.schedule.globs.hidden_states.device)
            self._flip = 0
        return True

    def fill(self):
        self.schedule.globs.barriers.fill_(self.barrier_fill_val)

    def replace_with_noops(self):
        self.schedule.globs.instructions.zero_()

    def run(self, input_ids: Tensor, pos_id: int) -> Tensor:
        globs = self.schedule.globs
        if self._fused_step():
            # embedding gather and argmax inside the megakernel; the output
            # token alternates between two buffers so that a step may read the
            # previous step's token while writing its own
            self.fill()
            globs.pos_id = pos_id
            out = self._tokens[self._flip]
            self._flip ^= 1
            ids = input_ids.reshape(-1)[:1]
            if ids.dtype != torch.int64:
                ids = ids.to(torch.int64)
            self.interpreter.interpret_step(globs, ids, self.model.model.embed_tokens.embed_tokens.weight, out)
            return out[0]
        if not self.skip_rest:
            emb = self.model.model.embed_tokens(BatchState(input_ids=input_ids))
            globs.hidden_states[:] = emb.hidden_states.reshape(-1)
        self.fill()
        globs.pos_id = pos_id
        globs.logits.zero_()
        if not self.skip_mk:
            self.interpreter.interpret(globs)
        if self.skip_rest:
            return input_ids
        return torch.argmax(globs.logits, dim=-1)

    def prefill(self, prompt_ids: Tensor, start_pos: int = 0) -> Tensor:
        """Fill the KV cache with the prompt (the model's dense prefill, as
        the reference's model forward does before MK decoding) and return the
        first generated token (argmax of the last prompt token's logits)."""
        logits = self.model.prefill(prompt_ids, start_pos)
        return torch.argmax(logits, dim=-1)

    def generate(self, output_tokens: Tensor, prompt_len: int, ntok: int,
                 ntok_already_generated: int = 1):
        for i in range(ntok):
            src = ntok_already_generated + i - 1
            input_ids = output_tokens[:, src : src + 1]
            out = self.run(input_ids, pos_id=prompt_len + ntok_already_generated + i - 1)
            output_tokens[:, src + 1] = out.reshape(-1)
