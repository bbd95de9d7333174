"""How the multi-GPU benchmark splits its work across ranks (host arithmetic only).

RNG: each step is curandGenerateUniform(n) then curandGenerateNormal(n)
on one generator.  Philox is counter-based, so ranks need no communication: rank r
sets its generator's offset to r * 2n words and draws the same two calls, covering
words [2rn, 2(r+1)n) of the single global stream (uniform block, then normal block).
The ranges of the ranks are disjoint and contiguous, and with n a multiple of 4 no
Philox block (4 words) is shared between ranks (the reference's offset rule,
curand_api.mm:117-125: block = word offset >> 2).
"""


def rng_rank_offset(rank: int, words_per_call: int) -> int:
    """Generator offset (in words) of `rank` for a uniform + normal step of
    `words_per_call` words each."""
    if rank < 0 or words_per_call < 0:
        raise ValueError("rank and words_per_call must be non-negative")
    return rank * 2 * words_per_call
