"""The planted-bug test of the host emulator (gemm-ladder_b200/emu/planted_bugs.py) stays runnable as the kernel's
sources change: every mutation's text is still where it names, in a build the script defines and has calls for, and
no two mutations share a name or an edit.  (The full run compiles one emulator per mutation and takes about half an
hour on 6 cores; its last record is gemm-ladder_b200/emu/planted_bugs.txt.)"""
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "gemm-ladder_b200", "emu"))

import planted_bugs as pb  # noqa: E402


def test_every_mutation_applies_to_the_current_sources():
    texts = {}
    for m in pb.MUTATIONS:
        name, rel, before, after, nth, build = m
        if rel not in texts:
            with open(os.path.join(ROOT, "gemm-ladder_b200", rel)) as f:
                texts[rel] = f.read()
        pb.locate(texts[rel], m)  # raises if the text is gone
        assert before != after, name
        assert build in pb.BUILDS and pb.CASES.get(build), f"{name}: build {build} has no calls"


def test_mutations_are_distinct_and_cover_every_build():
    names = [m[0] for m in pb.MUTATIONS]
    assert len(names) == len(set(names)), "two mutations share a name"
    edits = [(m[1], m[2], m[4], m[3]) for m in pb.MUTATIONS]
    assert len(edits) == len(set(edits)), "two mutations make the same edit"
    assert len(pb.MUTATIONS) >= 100
    assert {m[5] for m in pb.MUTATIONS} == set(pb.BUILDS), "a build without mutations, or a mutation without a build"
