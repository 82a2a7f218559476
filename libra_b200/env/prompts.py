"""Prompt templates of the workflows (our own wording)."""

MATH_SYSTEM = "Solve the problem step by step. Put the final answer inside \\boxed{} at the end."
MATH_USER = "{question}"

SEARCH_R1_SYSTEM = (
    "Answer the question. Think inside <think></think>. When you need facts, issue a query as "
    "<search>query</search>; results come back inside <information></information>. Search as often as needed, "
    "then give only the final answer as <answer>answer</answer>.")

R2E_ISSUE_SYSTEM = (
    "You are given a repository change and the tests it breaks. Write the GitHub issue a user would file: a "
    "title, the steps or code that reproduce it, the expected behaviour and the actual behaviour or error. "
    "Wrap the issue in [ISSUE] and [/ISSUE].")

CODE_AGENT_SYSTEM = (
    "Write a Python program that solves the task. You may test code by sending it in a ```python block; the "
    "execution result comes back to you. When you are done, send the final program in a ```python block "
    "followed by <submit>.")


def chat(tokenizer, messages, add_generation_prompt: bool = True) -> str:
    """Chat template when the tokenizer has one, else a plain role-tagged transcript."""
    if getattr(tokenizer, "chat_template", None):
        try:
            return tokenizer.apply_chat_template(messages, tokenize=False, add_generation_prompt=add_generation_prompt,
                                                 enable_thinking=False)
        except TypeError:
            return tokenizer.apply_chat_template(messages, tokenize=False, add_generation_prompt=add_generation_prompt)
    text = "".join(f"<|{m['role']}|>\n{m['content']}\n" for m in messages)
    return text + ("<|assistant|>\n" if add_generation_prompt else "")
