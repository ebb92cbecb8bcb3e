"""The table-driven SFT / eval datasets: rendered conversations and graders on in-memory rows."""

from mint_b200.data.datasets.catalog import (
    ARC,
    GSM8K,
    MMLU,
    CustomJSON,
    HumanEval,
    SimpleSpelling,
    SpellingBee,
    calculator_parts,
)


def test_multiple_choice_render_and_grade():
    arc = ARC(ds=[{"question": "Q?", "choices": {"text": ["a", "b"], "label": ["A", "B"]}, "answerKey": "B"}])
    conv = arc[0]
    assert conv["messages"][0]["content"] == (
        "Multiple Choice question: Q?\n- a=A\n- b=B\n\nRespond only with the letter of the correct answer.")
    assert conv["messages"][1] == {"role": "assistant", "content": "B"} and conv["letters"] == ("A", "B")
    assert arc.evaluate(conv, "B") and not arc.evaluate(conv, "A") and arc.eval_type == "categorical"
    mm = MMLU(ds=[{"question": "Q", "choices": ["w", "x", "y", "z"], "answer": 2, "subject": "s"}])
    assert mm[0]["messages"][1]["content"] == "C" and mm[0]["subject"] == "s"


def test_gsm8k_calculator_parts_and_answer():
    assert calculator_parts("a <<2*3=6>> b") == [
        {"type": "text", "text": "a "}, {"type": "python", "text": "2*3"},
        {"type": "python_output", "text": "6"}, {"type": "text", "text": " b"}]
    g = GSM8K(ds=[{"question": "q", "answer": "x <<1+1=2>>\n#### 1,234"}])
    assert g.evaluate(g[0], "so #### 1234") and not g.evaluate(g[0], "#### 12")


def test_spelling_tasks_are_reproducible():
    words = ["apple", "banana", "cherry"]
    a, b = SpellingBee(size=4, words=words), SpellingBee(size=4, words=words)
    assert [a[i] for i in range(4)] == [b[i] for i in range(4)]
    test = SpellingBee(size=4, split="test", words=words)
    assert [test[i] for i in range(4)] != [a[i] for i in range(4)]
    conv = a[1]
    assert a.evaluate(conv, conv["messages"][1]["content"][-1]["text"])
    s = SimpleSpelling(size=2, words=["cat", "dog"])
    word = s[0]["messages"][0]["content"].split(": ")[1]
    assert s[0]["messages"][1]["content"] == f"{word}:{','.join(word)}"


def test_humaneval_grades_by_running_tests():
    he = HumanEval(ds=[{"prompt": "import math\ndef f(x):\n", "canonical_solution": "    return math.sqrt(x)\n",
                        "entry_point": "f", "test": "def check(fn):\n    assert fn(4) == 2\n"}])
    good = "```python\ndef f(x):\n    return math.sqrt(x)\n```"
    assert he.evaluate(he[0], good)
    assert not he.evaluate(he[0], "def f(x):\n    return x")


def test_custom_jsonl(tmp_path):
    p = tmp_path / "c.jsonl"
    p.write_text('[{"role": "user", "content": "hi"}, {"role": "assistant", "content": "yo"}]\n\n')
    ds = CustomJSON(str(p))
    assert len(ds) == 1 and ds[0]["messages"][1]["content"] == "yo"
    assert len(CustomJSON(str(tmp_path / "missing.jsonl"))) == 0
