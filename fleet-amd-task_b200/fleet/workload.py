"""The benchmark configurations' seeded synthetic inputs, built on the device.

BASELINE.json's configs name seeded synthetic data (no checkpoint, no dataset):

* weights: BF16 ~N(0, 0.02) from seed 0, norm weights 1.0 (fleet.pack_weights.synthetic_packed);
* the prompt: token ids uniform over [0, V) from seed 2 (a CPU torch.Generator, so the ids do not
  depend on the device);
* the latent cache the prefill would leave: c_kv and k_pe rows ~N(0,1) BF16, seed 1 at config 1's
  1K context, seed 5 at config 4's 8K context (fleet.capture.make_capture).

`greedy_decode` builds all of that for a context of `n_prompt` tokens with room for `new_tokens`
greedy decode steps, so that the bench, the parity tests and the fixture scripts decode the same
tokens from the same state.
"""
from dataclasses import dataclass

import torch

from fleet.capture import make_capture
from fleet.pack_weights import REAL_DIMS, Dims, synthetic_packed

C1_PROMPT = 1024
WEIGHT_SEED, CACHE_SEED_1K, PROMPT_SEED, CACHE_SEED_8K = 0, 1, 2, 5


@dataclass
class Workload:
    dims: Dims
    packed: dict
    capture: dict
    prompt: list
    n_prompt: int
    s_max: int

    @property
    def first_pos(self):
        """Position of the first decode iteration: it reads the last prompt token and writes
        tokens[n_prompt]."""
        return self.n_prompt - 1


def prompt_ids(dims: Dims, n_prompt: int, seed: int = PROMPT_SEED):
    return torch.randint(0, dims.V, (n_prompt,), generator=torch.Generator().manual_seed(seed)).tolist()


def greedy_decode(device, n_prompt=C1_PROMPT, new_tokens=32, layers=None, dims: Dims = REAL_DIMS,
                  cache_seed=None, extra_rows=0):
    """Config 1 (n_prompt 1024) or config 4 (8192): the model, its cache of n_prompt - 1 prefilled
    rows, the prompt, and s_max = n_prompt + new_tokens + extra_rows."""
    layers = dims.L if layers is None else layers
    s_max = n_prompt + new_tokens + extra_rows
    if cache_seed is None:
        cache_seed = CACHE_SEED_1K if n_prompt <= C1_PROMPT else CACHE_SEED_8K
    packed = synthetic_packed(dims, layers=layers, head=True, seed=WEIGHT_SEED, device=device)
    capture = make_capture(dims, layers, s_max, n_prompt - 1, seed=cache_seed, device=device)
    return Workload(dims, packed, capture, prompt_ids(dims, n_prompt), n_prompt, s_max)
