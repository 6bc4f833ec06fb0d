"""Token loops around the megakernel (`megakernels/generators.py` of
epic-kernel, :11-166).

`MK_Generator.run` does per token what the reference does: embed the input
token into `hidden_states`, reset the barrier counters, zero the logits, launch
the megakernel, and take the argmax of the logits, all on the current stream
with no host synchronisation.
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

    def fill(self):
        self.schedule.globs.barriers.fill_(self.barrier_fill_val)

    def replace_with_noops(self):
        self.schedule.globs.instructions.zero_()

    def run(self, input_ids: Tensor, pos_id: int) -> Tensor:
        globs = self.schedule.globs
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

    def generate(self, output_tokens: Tensor, prompt_len: int, ntok: int,
                 ntok_already_generated: int = 1):
        for i in range(ntok):
            src = ntok_already_generated + i - 1
            input_ids = output_tokens[:, src : src + 1]
            out = self.run(input_ids, pos_id=prompt_len + ntok_already_generated + i - 1)
            output_tokens[:, src + 1] = out.reshape(-1)
