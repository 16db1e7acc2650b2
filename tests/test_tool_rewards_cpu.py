"""Verified tool episodes and completion rewards (CPU)."""
import pytest

from complexity_framework_b200.rl import tool_rewards as tr


def test_calculator_episode_and_safety():
    ep = tr.build_verified_tool_episode("P", "What is 12 * (3 + 4)?")
    assert ep.tool_call == {"name": "calculator", "arguments": {"expression": "12*(3+4)"}}
    assert ep.target_response == ('<tool_call>{"name":"calculator","arguments":'
                                  '{"expression":"12*(3+4)"}}</tool_call>\n'
                                  "Tool result from calculator: 84\nAssistant:\n84")
    assert tr.safe_calculator("7/2") == "3.5" and tr.safe_calculator("8/2") == "4"
    for bad in ("2**100", "1/0", "__import__('os')", "(1+"):
        with pytest.raises(tr.CalculatorError):
            tr.safe_calculator(bad)
    assert tr.extract_arithmetic_expression("hello there") is None


def test_datetime_episodes():
    ep = tr.build_verified_tool_episode("P", "What day of the week is 2024-03-01?")
    assert ep.tool_result["result"] == "Friday"
    ep = tr.build_verified_tool_episode("P", "Days between 2024-01-01 and 2024-03-01?")
    assert ep.tool_result["result"] == "60"
    ep = tr.build_verified_tool_episode("P", "What is 2024-02-27 plus 3 days?")
    assert ep.tool_result["result"] == "2024-03-01"
    assert '"op":"add_days","date":"2024-02-27","days":3' in ep.target_response
    with pytest.raises(tr.DatetimeError):
        tr.safe_datetime("weekday", date="2024-13-01")


def test_reward_scores_completions():
    ep = tr.build_verified_tool_episode("P", "calculate 6*7")
    assert tr.tool_call_reward(ep.target_response, ep) == pytest.approx(1.0)
    wrong_call = ep.target_response.replace("6*7", "6*8")
    assert tr.tool_call_reward(wrong_call, ep) == pytest.approx(0.2 + 0.4)
    assert tr.tool_call_reward("42", ep) == pytest.approx(0.4)
    assert tr.tool_call_reward("<tool_call>{bad json</tool_call> 41", ep) == 0.0
    assert tr.batch_tool_rewards([ep.target_response, "no"], ep) == [pytest.approx(1.0), 0.0]
