"""The numerics-identity payload (no GPU): the behaviours the reference's own
conformance test checks (tests/numerics_identity_tests.cpp), and byte-for-byte
agreement with the reference's implementation (src/bitstream/numerics_identity.cpp,
compiled into oracle/_ref) on seeded random stage lists and payloads, valid and
invalid."""
from __future__ import annotations

import random

import pytest

from nvcr_b200.executor import ErrorCode, ExecutorError, numerics_identity, parse_numerics_identity

PROFILE = "nvcr.intconv.v1"


def sample_stages():
    stages = []
    for name in ("i_hyper_synthesis", "i_synthesis", "p_prior", "p_synthesis"):
        stages.append((name, bytes(((i * 37 + len(name)) & 0xFF) for i in range(32))))
    return stages


def error_code(call) -> ErrorCode:
    with pytest.raises(ExecutorError) as raised:
        call()
    return raised.value.code


def test_round_trip():
    payload = numerics_identity(PROFILE, sample_stages())
    assert len(payload) == 1 + len(PROFILE) + 32
    assert payload[0] == len(PROFILE) and payload[1:1 + len(PROFILE)] == PROFILE.encode()
    profile, digest = parse_numerics_identity(payload)
    assert profile == PROFILE and digest == payload[-32:]


def test_program_set_digest_covers_every_part():
    stages = sample_stages()
    base = numerics_identity(PROFILE, stages)
    assert numerics_identity(PROFILE, stages) == base  # deterministic
    flipped = list(stages)
    digest = bytearray(flipped[2][1])
    digest[31] ^= 1
    flipped[2] = (flipped[2][0], bytes(digest))
    renamed = list(stages)
    renamed[1] = ("i_synthesis2", renamed[1][1])
    swapped = [stages[1], stages[0]] + stages[2:]
    for variant in (numerics_identity(PROFILE, flipped), numerics_identity(PROFILE, renamed),
                    numerics_identity(PROFILE, swapped)):
        assert variant[-32:] != base[-32:]  # the program-set digest changes
    other = numerics_identity("nvcr.other.v1", stages)
    assert other != base and other[-32:] == base[-32:]  # the profile is part of the identity, not of the digest


def test_truncation_and_trailing_bytes_are_malformed():
    payload = numerics_identity(PROFILE, sample_stages())
    for length in range(len(payload)):
        assert error_code(lambda: parse_numerics_identity(payload[:length])) == ErrorCode.malformed_bitstream
    assert error_code(lambda: parse_numerics_identity(payload + b"\0")) == ErrorCode.malformed_bitstream


def test_invalid_contents():
    stages = sample_stages()
    duplicate = [stages[0], (stages[0][0], stages[1][1])] + stages[2:]
    assert error_code(lambda: numerics_identity(PROFILE, duplicate)) == ErrorCode.invalid_argument
    assert error_code(lambda: numerics_identity(PROFILE, [])) == ErrorCode.invalid_argument
    assert error_code(lambda: numerics_identity("nvcr intconv.v1", stages)) == ErrorCode.invalid_argument
    too_many = [(f"s{i}", bytes(32)) for i in range(65)]
    assert error_code(lambda: numerics_identity(PROFILE, too_many)) == ErrorCode.invalid_argument
    assert len(numerics_identity(PROFILE, too_many[:64])) == 1 + len(PROFILE) + 32
    assert error_code(lambda: numerics_identity("x" * 129, stages)) == ErrorCode.invalid_argument
    control = bytes([1, 0x07]) + bytes(32)
    assert error_code(lambda: parse_numerics_identity(control)) == ErrorCode.malformed_bitstream
    empty_profile = bytes([0]) + bytes(32)
    assert error_code(lambda: parse_numerics_identity(empty_profile)) == ErrorCode.malformed_bitstream


def random_id(rng: random.Random) -> str:
    kind = rng.random()
    if kind < 0.05:
        return ""
    if kind < 0.1:
        return "a" * 129
    if kind < 0.15:
        return "bad id"
    if kind < 0.2:
        return "ctl\x1f"
    return "".join(chr(rng.randint(0x21, 0x7E)) for _ in range(rng.randint(1, 128 if kind < 0.25 else 12)))


def ours_or_code(call):
    try:
        return 0, call()
    except ExecutorError as error:
        return int(error.code) + 1, None


def test_stage_lists_match_the_reference(reference):
    rng = random.Random(216)
    for _ in range(300):
        count = rng.choice([0, 1, 2, 5, 64, 65]) if rng.random() < 0.2 else rng.randint(1, 8)
        stages = [(random_id(rng) if rng.random() < 0.3 else f"stage_{rng.randint(0, 9)}",
                   bytes(rng.getrandbits(8) for _ in range(32))) for _ in range(count)]
        profile = random_id(rng) if rng.random() < 0.3 else PROFILE
        expected_status, expected = reference.numerics_identity(profile, stages)
        status, got = ours_or_code(lambda: numerics_identity(profile, stages))
        assert status == expected_status, (profile, [s for s, _ in stages])
        if status == 0:
            assert got == expected


def test_payloads_match_the_reference(reference):
    rng = random.Random(217)
    valid = numerics_identity(PROFILE, sample_stages())
    for _ in range(500):
        kind = rng.random()
        if kind < 0.3:
            payload = bytearray(valid)
            for _ in range(rng.randint(1, 3)):
                payload[rng.randrange(len(payload))] = rng.getrandbits(8)
        elif kind < 0.6:
            payload = bytearray(valid[:rng.randint(0, len(valid))] + bytes(rng.getrandbits(8)
                                                                          for _ in range(rng.randint(0, 3))))
        else:
            length = rng.randint(0, 140)
            payload = bytearray([length]) + bytes(rng.randint(0x10, 0x80) for _ in range(length)) + \
                bytes(rng.getrandbits(8) for _ in range(rng.choice([31, 32, 33])))
        payload = bytes(payload)
        expected = reference.parse_numerics_identity(payload)
        status, got = ours_or_code(lambda: parse_numerics_identity(payload))
        assert status == expected[0], payload
        if status == 0:
            assert got == (expected[1], expected[2])
